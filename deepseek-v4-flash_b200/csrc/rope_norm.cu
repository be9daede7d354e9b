// rope_norm.cu -- per-head RMSNorm and rotary embedding on bf16 rows.
//
//  * RMSNorm follows Deepseek_origin/inference/model.py:498
//    (`q *= rsqrt(q.square().mean(-1) + eps)` on a bf16 tensor) and
//    QCAU/QCAU_inference/inference/QCAU.py:16-27 (optional per-head gamma):
//    every elementwise step rounds to bf16, the mean accumulates in fp32.
//  * RoPE follows model.py:231-243 / QCAU.py:30-68: the last rope_dim values
//    of a row are interleaved (re, im) pairs multiplied by freqs_cis[pos]
//    (its conjugate for the inverse) in fp32, stored as bf16.
//
// One warp per row; lanes own consecutive value pairs, so loads are
// coalesced 4-byte accesses and a RoPE pair never straddles two lanes.
#include "common.cuh"
#include "kernels.h"

namespace qcau {

__global__ void head_norm_rope_kernel(__nv_bfloat16* __restrict__ q,
                                      const __nv_bfloat16* __restrict__ gamma,
                                      const float* __restrict__ freqs,
                                      const int32_t* __restrict__ positions, int64_t rows,
                                      int64_t seqlen, int64_t heads, int d, int64_t row_stride,
                                      int rope_dim, int64_t pos0, float eps, int do_norm,
                                      int do_rope, int inverse) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t bt = r / heads, h = r % heads;
  __nv_bfloat162* row = reinterpret_cast<__nv_bfloat162*>(q + r * row_stride);
  const int npairs = d / 2;
  constexpr int kMaxPairsPerLane = 16;  // d <= 1024
  float2 v[kMaxPairsPerLane];
#pragma unroll
  for (int k = 0; k < kMaxPairsPerLane; k++) {
    const int j = lane + 32 * k;
    if (j < npairs) v[k] = __bfloat1622float2(row[j]);
  }
  if (do_norm) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxPairsPerLane; k++) {
      const int j = lane + 32 * k;
      if (j < npairs) acc += bf16_round(v[k].x * v[k].x) + bf16_round(v[k].y * v[k].y);
    }
    acc = warp_sum(acc);
    const float mean = bf16_round(__fdiv_rn(acc, (float)d));
    const float rs = bf16_round(__frcp_rn(__fsqrt_rn(bf16_round(mean + eps))));
    const __nv_bfloat162* g =
        gamma ? reinterpret_cast<const __nv_bfloat162*>(gamma + h * d) : nullptr;
#pragma unroll
    for (int k = 0; k < kMaxPairsPerLane; k++) {
      const int j = lane + 32 * k;
      if (j < npairs) {
        v[k].x = bf16_round(v[k].x * rs);
        v[k].y = bf16_round(v[k].y * rs);
        if (g) {
          float2 gg = __bfloat1622float2(g[j]);
          v[k].x = bf16_round(v[k].x * gg.x);
          v[k].y = bf16_round(v[k].y * gg.y);
        }
      }
    }
  }
  if (do_rope) {
    const int64_t b = bt / seqlen, t = bt % seqlen;
    const int64_t pos = positions ? (int64_t)positions[b * seqlen + t] : pos0 + t;
    const float2* f = reinterpret_cast<const float2*>(freqs) + pos * (rope_dim / 2);
    const int first = (d - rope_dim) / 2;
#pragma unroll
    for (int k = 0; k < kMaxPairsPerLane; k++) {
      const int j = lane + 32 * k;
      if (j < npairs && j >= first) {
        const float2 cs = f[j - first];
        const float sn = inverse ? -cs.y : cs.y;
        const float a = v[k].x, bb = v[k].y;
        v[k].x = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(bb, sn));
        v[k].y = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(bb, cs.x));
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kMaxPairsPerLane; k++) {
    const int j = lane + 32 * k;
    if (j < npairs) row[j] = __floats2bfloat162_rn(v[k].x, v[k].y);
  }
}

cudaError_t launch_head_norm_rope(void* q, const void* gamma, const float* freqs,
                                  const int32_t* positions, int64_t b, int64_t s, int64_t h,
                                  int d, int64_t row_stride, int rope_dim, int64_t pos0,
                                  float eps, int do_norm, int do_rope, int inverse,
                                  cudaStream_t st) {
  const int64_t rows = b * s * h;
  if (rows == 0) return cudaSuccess;
  if (d > 1024 || (d & 1)) return cudaErrorInvalidValue;
  const int warps = 8;
  head_norm_rope_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, st>>>(
      reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(gamma), freqs,
      positions, rows, s, h, d, row_stride, rope_dim, pos0, eps, do_norm, do_rope, inverse);
  return cudaGetLastError();
}

// RoPE of the rope part only: one thread per (re, im) pair of a row, the
// rotated pair written back in place and, when `copy` is given, also to the
// matching pair of another row layout (the absorbed query's rope slot), so
// that the rope part is read once.  Same arithmetic as head_norm_rope_kernel.
__global__ void rope_pairs_kernel(__nv_bfloat16* __restrict__ x, int64_t x_stride,
                                  __nv_bfloat16* __restrict__ copy, int64_t copy_stride,
                                  const float* __restrict__ freqs,
                                  const int32_t* __restrict__ positions, int64_t rows,
                                  int64_t seqlen, int64_t heads, int pairs, int64_t pos0,
                                  int inverse) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * pairs) return;
  const int64_t r = i / pairs;
  const int j = (int)(i % pairs);
  const int64_t bt = r / heads, b = bt / seqlen, t = bt % seqlen;
  const int64_t pos = positions ? (int64_t)positions[b * seqlen + t] : pos0 + t;
  const float2 cs = reinterpret_cast<const float2*>(freqs)[pos * pairs + j];
  const float sn = inverse ? -cs.y : cs.y;
  __nv_bfloat162* px = reinterpret_cast<__nv_bfloat162*>(x + r * x_stride) + j;
  const float2 v = __bfloat1622float2(*px);
  const __nv_bfloat162 o = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(v.x, cs.x), __fmul_rn(v.y, sn)),
                                                 __fadd_rn(__fmul_rn(v.x, sn), __fmul_rn(v.y, cs.x)));
  *px = o;
  if (copy) reinterpret_cast<__nv_bfloat162*>(copy + r * copy_stride)[j] = o;
}

cudaError_t launch_rope_pairs(void* x, int64_t x_stride, void* copy, int64_t copy_stride,
                              const float* freqs, const int32_t* positions, int64_t b, int64_t s,
                              int64_t h, int rope_dim, int64_t pos0, int inverse,
                              cudaStream_t st) {
  const int64_t rows = b * s * h;
  if (rows == 0) return cudaSuccess;
  if (rope_dim <= 0 || (rope_dim & 1)) return cudaErrorInvalidValue;
  const int pairs = rope_dim / 2;
  const int64_t n = rows * pairs;
  rope_pairs_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<__nv_bfloat16*>(x), x_stride, reinterpret_cast<__nv_bfloat16*>(copy),
      copy_stride, freqs, positions, rows, s, h, pairs, pos0, inverse);
  return cudaGetLastError();
}

}  // namespace qcau
