// kv_build.cu -- the latent KV row of a new token, from the wkv projection to
// the cache (Deepseek_origin/inference/model.py:502-506 and the cache writes
// :517-533):
//   kv = kv_norm(kv)                      RMSNorm in fp32 with an fp32 weight,
//                                         stored as bf16 (model.py:182-195)
//   kv[..., -rd:] = RoPE(kv[..., -rd:])   interleaved pairs times
//                                         freqs_cis[pos] in fp32 (:231-243)
//   act_quant(kv[..., :-rd], 64, fmt, inplace=True)
//                                         the FP8 round trip of the non-rope
//                                         values: 1 x 64 blocks, e4m3 codes
//                                         and back to bf16 (kernel.py:40-125)
//   kv_cache[slot] = kv                   the window ring (slot = pos % win,
//                                         model.py:517-526, :530) or a paged
//                                         cache (slot = page * 64 + pos % 64)
// For the absorbed-MLA cache row (512 latent + 64 rope) the norm covers the
// first 512 values and there is no FP8 round trip.
//
// One warp per row (HBM-bound byte work): lane l holds values 64k + 2l,
// 64k + 2l + 1 of every 64-value block k, so a quantisation block is one
// warp-wide max, a RoPE pair never straddles lanes, and every load and store
// of the warp is a coalesced 128-byte run.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kMaxBlocks = 16;  // d <= 1024

__global__ void __launch_bounds__(256) kv_build_kernel(KvBuildArgs p, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= p.rows) return;
  const int nb = (int)(p.d / 64);
  const __nv_bfloat162* in = reinterpret_cast<const __nv_bfloat162*>(p.in) + r * (p.d / 2);
  float2 v[kMaxBlocks];
#pragma unroll
  for (int k = 0; k < kMaxBlocks; k++)
    if (k < nb) v[k] = __bfloat1622float2(in[32 * k + lane]);

  // RMSNorm over [0, norm_dim): fp32 squares and mean, x * rsqrt(var + eps),
  // then times the weight, rounded to bf16 once (model.py:190-195)
  if (p.norm_dim > 0) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxBlocks; k++)
      if (64 * k < p.norm_dim) acc += __fmul_rn(v[k].x, v[k].x) + __fmul_rn(v[k].y, v[k].y);
    acc = warp_sum(acc);
    // 1 / sqrt, two correctly rounded steps: torch's rsqrt on the CPU
    const float rs = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)p.norm_dim), p.eps)));
#pragma unroll
    for (int k = 0; k < kMaxBlocks; k++) {
      if (64 * k < p.norm_dim) {
        const int dim = 64 * k + 2 * lane;
        const float w0 = p.norm_weight ? p.norm_weight[dim] : 1.f;
        const float w1 = p.norm_weight ? p.norm_weight[dim + 1] : 1.f;
        v[k].x = bf16_round(__fmul_rn(w0, __fmul_rn(v[k].x, rs)));
        v[k].y = bf16_round(__fmul_rn(w1, __fmul_rn(v[k].y, rs)));
      }
    }
  }

  // RoPE of the last rope_dim values at this row's position
  const int64_t seq = p.seq_rows > 0 ? r / p.seq_rows : 0;
  const int64_t i_new = p.seq_rows > 0 ? r - seq * p.seq_rows : 0;
  if (p.rope_dim > 0) {
    const int64_t pos = p.seq_rows > 0 ? p.pos_base + i_new * p.pos_step : p.positions[r];
    if (pos < 0 || pos >= p.npos) {
      if (lane == 0) raise_dev_error(err, QCAU_DEVERR_INDEX);
    } else {
      const float2* f = reinterpret_cast<const float2*>(p.freqs) + pos * (p.rope_dim / 2);
      const int first = (int)p.d - p.rope_dim;
#pragma unroll
      for (int k = 0; k < kMaxBlocks; k++) {
        const int dim = 64 * k + 2 * lane;
        if (k < nb && dim >= first) {
          const float2 cs = f[(dim - first) / 2];
          const float a = v[k].x, b = v[k].y;
          v[k].x = bf16_round(__fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y)));
          v[k].y = bf16_round(__fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x)));
        }
      }
    }
  }

  // FP8 round trip of the blocks below quant_dims
#pragma unroll
  for (int k = 0; k < kMaxBlocks; k++) {
    if (64 * k < p.quant_dims) {
      const float amax = warp_max(fmaxf(fabsf(v[k].x), fabsf(v[k].y)));
      const float sc = act_scale(amax, p.round_scale);
      float q0, q1;
      if (p.round_scale) {
        // sc = 2^e with -22 <= e <= 120: x * 2^-e is the exact quotient
        // rounded once, the same number __fdiv_rn gives
        const float inv = __uint_as_float((uint32_t)(254 - (int)(__float_as_uint(sc) >> 23)) << 23);
        q0 = __fmul_rn(v[k].x, inv);
        q1 = __fmul_rn(v[k].y, inv);
      } else {
        q0 = __fdiv_rn(v[k].x, sc);
        q1 = __fdiv_rn(v[k].y, sc);
      }
      q0 = fminf(fmaxf(q0, -448.f), 448.f);
      q1 = fminf(fmaxf(q1, -448.f), 448.f);
      v[k].x = bf16_round(__fmul_rn(e4m3_to_f32(f32_to_e4m3(q0)), sc));
      v[k].y = bf16_round(__fmul_rn(e4m3_to_f32(f32_to_e4m3(q1)), sc));
    }
  }

  __nv_bfloat162* out = p.out ? reinterpret_cast<__nv_bfloat162*>(p.out) + r * (p.d / 2) : nullptr;
  int64_t slot = p.seq_rows > 0 && p.cache ? seq * p.slot_seq_stride + p.slot_base + i_new
                 : p.slots ? (int64_t)p.slots[r] : -1;
  if (slot >= p.cache_rows) {
    if (lane == 0) raise_dev_error(err, QCAU_DEVERR_INDEX);
    slot = -1;
  }
  __nv_bfloat162* dst = slot >= 0 ? reinterpret_cast<__nv_bfloat162*>(p.cache) + slot * (p.d / 2)
                                  : nullptr;
#pragma unroll
  for (int k = 0; k < kMaxBlocks; k++) {
    if (k < nb) {
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[k].x, v[k].y);
      if (out) out[32 * k + lane] = b2;
      if (dst) dst[32 * k + lane] = b2;
    }
  }
}

}  // namespace

cudaError_t launch_kv_build(const KvBuildArgs& a, cudaStream_t st) {
  if (a.rows == 0) return cudaSuccess;
  if (a.d % 64 || a.d > 64 * kMaxBlocks) return cudaErrorInvalidValue;
  const int warps = 8;
  kv_build_kernel<<<(unsigned)((a.rows + warps - 1) / warps), warps * 32, 0, st>>>(
      a, device_error_word());
  return cudaGetLastError();
}

}  // namespace qcau
