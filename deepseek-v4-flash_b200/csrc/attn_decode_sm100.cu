// attn_decode_sm100.cu -- tcgen05 two-CTA paged decode attention (placeholder
// until the kernel lands: reports "unsupported" so the general kernel runs).
#include "common.cuh"
#include "kernels.h"

namespace qcau {

bool decode_attn_sm100_supported(const AttnArgs&) { return false; }

cudaError_t launch_decode_attn_sm100(const AttnArgs&, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace qcau
