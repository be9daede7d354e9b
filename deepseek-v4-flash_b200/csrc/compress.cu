// compress.cu -- the KV compressor's gated pooling
// (QCAU/QCAU_inference/inference/model.py:376-476, Compressor.forward; the
// same code is Deepseek_origin/inference/model.py:278-377).
//
// Every `ratio` consecutive tokens become one compressed row: per channel,
// the window's kv values weighted by the softmax of their gate scores (plus
// the learned position bias `ape`).  With overlap (ratio 4) the projections
// are 2d wide and a window holds 2 * ratio entries: the previous group's
// tokens on channels [0, d) and the current group's on channels [d, 2d)
// (overlap_transform, model.py:406-413; the first group's previous half is
// value 0 / score -inf).  Arithmetic is fp32 as the reference's (x.float()),
// the softmax max-subtracted, the weighted sum over the window in order, and
// the pooled row rounded to bf16 (kv.to(dtype), model.py:459) for the norm,
// RoPE and quantisation that follow (kv_build.cu).
//
// Prefill (start_pos 0): pooled rows of the seqlen // ratio complete groups,
// and the decode state the reference leaves behind: the last complete group
// (overlap) and the remainder tokens.  Decode (one token): the token's kv and
// biased score go into the state; at a group boundary ((start_pos + 1) %
// ratio == 0) the state is pooled, and with overlap shifted by one group.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kMaxWin = 2 * 128;  // entries of one window (2 * ratio with overlap)

// softmax-weighted sum over the w entries entry(j) -> (kv_j, score_j), in
// entry order; the entries are read again in each pass instead of held
template <class Entry>
__device__ __forceinline__ float pool_window(Entry entry, int w) {
  float m = -INFINITY;
#pragma unroll 8
  for (int j = 0; j < w; j++) {
    float k, sc;
    entry(j, k, sc);
    m = fmaxf(m, sc);
  }
  if (m == -INFINITY) return 0.f;  // cannot happen: the current group's scores are finite
  float sum = 0.f;
#pragma unroll 8
  for (int j = 0; j < w; j++) {
    float k, sc;
    entry(j, k, sc);
    sum += expf(sc - m);
  }
  float acc = 0.f;
#pragma unroll 8
  for (int j = 0; j < w; j++) {
    float k, sc;
    entry(j, k, sc);
    acc += k * (expf(sc - m) / sum);
  }
  return acc;
}

// The same pooling with the window's W entries loaded into registers first,
// so their loads are in flight together instead of one after another (the
// ratio-4 compressors: W = 8 with overlap, 4 without).  Same arithmetic, in
// the same order, as pool_window.
template <int W, class Entry>
__device__ __forceinline__ float pool_window_regs(Entry entry) {
  float k[W], sc[W];
#pragma unroll
  for (int j = 0; j < W; j++) entry(j, k[j], sc[j]);
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < W; j++) m = fmaxf(m, sc[j]);
  if (m == -INFINITY) return 0.f;
  float e[W], sum = 0.f;
#pragma unroll
  for (int j = 0; j < W; j++) {
    e[j] = expf(sc[j] - m);
    sum += e[j];
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < W; j++) acc += k[j] * (e[j] / sum);
  return acc;
}

template <int W, class Entry>
__device__ __forceinline__ float pool(Entry entry, int w) {
  if constexpr (W > 0) {
    return pool_window_regs<W>(entry);
  } else {
    return pool_window(entry, w);
  }
}

// One thread per (sequence, group, channel c < d); W = the window's entries
// when known at compile time, else 0.
template <int W>
__global__ void compress_prefill_kernel(const float* __restrict__ kv, const float* __restrict__ score,
                                        const float* __restrict__ ape, __nv_bfloat16* __restrict__ out,
                                        int64_t bsz, int64_t seqlen, int d, int ratio, int overlap) {
  const int64_t groups = seqlen / ratio;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bsz * groups * d) return;
  const int c = (int)(i % d);
  const int64_t g = (i / d) % groups;
  const int64_t b = i / (d * groups);
  const int cw = overlap ? 2 * d : d;  // projection width
  const float* kvb = kv + b * seqlen * cw;
  const float* scb = score + b * seqlen * cw;
  const int ch = overlap ? d + c : c;
  auto entry = [&](int j, float& k, float& sc) {
    if (overlap && j < ratio) {  // the previous group, channels [0, d)
      if (g == 0) {
        k = 0.f;
        sc = -INFINITY;
      } else {
        const int64_t t = (g - 1) * ratio + j;
        k = kvb[t * cw + c];
        sc = scb[t * cw + c] + ape[j * cw + c];
      }
      return;
    }
    const int jj = overlap ? j - ratio : j;
    const int64_t t = g * ratio + jj;
    k = kvb[t * cw + ch];
    sc = scb[t * cw + ch] + ape[jj * cw + ch];
  };
  const float v = pool<W>(entry, overlap ? 2 * ratio : ratio);
  out[(b * groups + g) * d + c] = __float2bfloat16_rn(v);
}

// The state a prefill leaves (model.py:422-429): slots [0, ratio) <- the last
// complete group (overlap only), slots [off, off + rem) <- the remainder
// tokens (off = ratio with overlap, else 0); scores with ape added.  One
// thread per (sequence, slot, channel of the projection).
__global__ void compress_state_prefill_kernel(const float* __restrict__ kv,
                                              const float* __restrict__ score,
                                              const float* __restrict__ ape,
                                              float* __restrict__ kv_state,
                                              float* __restrict__ score_state, int64_t bsz,
                                              int64_t seqlen, int d, int ratio, int overlap) {
  const int cw = overlap ? 2 * d : d;
  const int slots = overlap ? 2 * ratio : ratio;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bsz * slots * cw) return;
  const int ch = (int)(i % cw);
  const int slot = (int)((i / cw) % slots);
  const int64_t b = i / ((int64_t)cw * slots);
  const int64_t rem = seqlen % ratio, cutoff = seqlen - rem;
  int64_t t = -1;
  int jape = 0;
  if (overlap && slot < ratio) {
    if (cutoff >= ratio) {
      t = cutoff - ratio + slot;
      jape = slot;
    }
  } else {
    const int off = overlap ? ratio : 0;
    if (slot - off < rem) {
      t = cutoff + (slot - off);
      jape = slot - off;
    }
  }
  if (t < 0) return;  // slot left as it was
  const int64_t src = (b * seqlen + t) * cw + ch;
  const int64_t dst = (b * slots + slot) * cw + ch;
  kv_state[dst] = kv[src];
  score_state[dst] = score[src] + ape[jape * cw + ch];
}

// One decode token per sequence (model.py:441-457): one thread per
// (sequence, channel c < d), which owns channels c and d + c of the state.
template <int W>
__global__ void compress_decode_kernel(const float* __restrict__ kv, const float* __restrict__ score,
                                       const float* __restrict__ ape, float* __restrict__ kv_state,
                                       float* __restrict__ score_state,
                                       __nv_bfloat16* __restrict__ out, int64_t bsz, int d, int ratio,
                                       int overlap, int64_t start_pos) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bsz * d) return;
  const int c = (int)(i % d);
  const int64_t b = i / d;
  const int cw = overlap ? 2 * d : d;
  const int slots = overlap ? 2 * ratio : ratio;
  const int p = (int)(start_pos % ratio);
  float* ks = kv_state + b * slots * cw;
  float* ss = score_state + b * slots * cw;
  const float* kvb = kv + b * cw;
  const float* scb = score + b * cw;
  const int slot = overlap ? ratio + p : p;
  for (int h = 0; h < (overlap ? 2 : 1); h++) {
    const int ch = c + h * d;
    ks[slot * cw + ch] = kvb[ch];
    ss[slot * cw + ch] = scb[ch] + ape[p * cw + ch];
  }
  if ((start_pos + 1) % ratio != 0) return;
  // overlap: cat(state[:ratio, :d], state[ratio:, d:]) (model.py:448-449)
  auto entry = [&](int j, float& k, float& sc) {
    const int ch = overlap && j >= ratio ? d + c : c;
    k = ks[j * cw + ch];
    sc = ss[j * cw + ch];
  };
  out[b * d + c] = __float2bfloat16_rn(pool<W>(entry, overlap ? 2 * ratio : ratio));
  if (overlap) {  // state[:ratio] = state[ratio:] (model.py:451-452)
#pragma unroll 4
    for (int j = 0; j < ratio; j++)
      for (int h = 0; h < 2; h++) {
        const int ch = c + h * d;
        ks[j * cw + ch] = ks[(ratio + j) * cw + ch];
        ss[j * cw + ch] = ss[(ratio + j) * cw + ch];
      }
  }
}

}  // namespace

cudaError_t launch_compress(const float* kv, const float* score, const float* ape, float* kv_state,
                            float* score_state, void* out, int64_t bsz, int64_t seqlen, int d,
                            int ratio, int overlap, int64_t start_pos, cudaStream_t st) {
  const int w = overlap ? 2 * ratio : ratio;
  if (ratio <= 0 || w > kMaxWin) return cudaErrorInvalidValue;
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  if (start_pos == 0) {
    const int64_t n = bsz * (seqlen / ratio) * d;
    if (n > 0) {
      const unsigned grid = (unsigned)((n + 127) / 128);
      auto kern = w == 8 ? compress_prefill_kernel<8>
                  : w == 4 ? compress_prefill_kernel<4> : compress_prefill_kernel<0>;
      kern<<<grid, 128, 0, st>>>(kv, score, ape, o, bsz, seqlen, d, ratio, overlap);
    }
    const int64_t ns = bsz * (int64_t)w * (overlap ? 2 * d : d);
    if (ns > 0 && kv_state)
      compress_state_prefill_kernel<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(
          kv, score, ape, kv_state, score_state, bsz, seqlen, d, ratio, overlap);
    return cudaGetLastError();
  }
  if (seqlen != 1) return cudaErrorInvalidValue;
  const int64_t n = bsz * d;
  if (n > 0) {
    auto kern = w == 8 ? compress_decode_kernel<8>
                : w == 4 ? compress_decode_kernel<4> : compress_decode_kernel<0>;
    kern<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(kv, score, ape, kv_state, score_state, o,
                                                      bsz, d, ratio, overlap, start_pos);
  }
  return cudaGetLastError();
}

}  // namespace qcau
