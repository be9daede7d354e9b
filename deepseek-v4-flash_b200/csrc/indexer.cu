// indexer.cu -- the producers of the top-k index lists that the sparse
// attention reads (QCAU/QCAU_inference/inference/model.py:302-376, :500-534;
// line numbers below are that file's):
//
//  * rotate_fp4: the indexer's score scaling of its query and key rows,
//    model.py:512-514 / :466-468: rotate_activation (a Walsh-Hadamard
//    transform scaled by d^-1/2: the third-party fast_hadamard_transform,
//    or the reference's own restatement of it, model.py:302-323, which is
//    what this follows bit for bit) and fp4_act_quant(x, 32, inplace=True)
//    (Deepseek_origin/inference/kernel.py:128-200): per 1x32 block
//    s = 2^ceil(log2(max(amax, 6*2^-126) * (1/6))), values
//    rounded to FP4 e2m1 {0, .5, 1, 1.5, 2, 3, 4, 6} (nearest, ties to even)
//    times s, back to bf16.  One warp per row of 128 values (4 a lane).
//  * index_score: the weighted ReLU sum of the raw scores (model.py:518-519):
//    score[b, s, t] = bf16(sum_h bf16(relu(raw[b, s, h, t]) * w[b, s, h])),
//    raw being the bf16 einsum q . kv (computed by the tcgen05 batched GEMM
//    of bmm.cu).
//  * topk: the top k of each score row (model.py:527) under the prefill
//    mask (:522-526), by a radix select over order-preserving keys (3 passes
//    of 11, 11 and 10 bits, one CTA a row), then a bitonic sort of the
//    selection by (score desc, index asc); -1 fills rows with fewer than k
//    candidates, where the reference's mask (:528-531) turns the -inf picks
//    into -1.
//  * index_lists: get_window_topk_idxs / get_compress_topk_idxs
//    (model.py:326-376), or the indexer's list in place of the latter,
//    concatenated as Attention.forward does (:614-624) into one [B, S, W]
//    list.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

// ---------------------------------------------------------------- rotate + FP4

// FP4 e2m1 value nearest to x (|x| <= 6), ties to the even code.
__device__ __forceinline__ float e2m1_round(float x) {
  const float a = fabsf(x);
  // code values 0, .5, 1, 1.5, 2, 3, 4, 6 with midpoints .25 .75 1.25 1.75 2.5 3.5 5
  float r;
  if (a <= 0.25f) r = 0.f;           // tie .25 -> 0 (code 0 even)
  else if (a < 0.75f) r = 0.5f;
  else if (a <= 1.25f) r = 1.f;      // tie .75 -> 1 (code 2), tie 1.25 -> 1 (code 2)
  else if (a < 1.75f) r = 1.5f;
  else if (a <= 2.5f) r = 2.f;       // tie 1.75 -> 2 (code 4), tie 2.5 -> 2 (code 4)
  else if (a < 3.5f) r = 3.f;
  else if (a <= 5.f) r = 4.f;        // tie 3.5 -> 4 (code 6), tie 5 -> 4 (code 6)
  else r = 6.f;
  return copysignf(r, x);
}

__global__ void __launch_bounds__(256) rotate_fp4_kernel(__nv_bfloat16* __restrict__ x, int64_t rows,
                                                         int hadamard, int fp4) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  // lane l holds values 4l .. 4l+3 (a block of 32 = 8 lanes)
  uint2 raw = reinterpret_cast<const uint2*>(x + r * 128)[lane];
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; i++) v[i] = __bfloat162float(h[i]);
  if (hadamard) {
    // Sylvester order: stage with span m pairs indices i, i + m (i & m == 0)
    // as (a + b, a - b); spans 1, 2 within the lane, 4..64 across lanes
#pragma unroll
    for (int m = 1; m <= 2; m <<= 1)
#pragma unroll
      for (int i = 0; i < 4; i++)
        if ((i & m) == 0) {
          const float a = v[i], b = v[i + m];
          v[i] = a + b;
          v[i + m] = a - b;
        }
#pragma unroll
    for (int lm = 1; lm <= 16; lm <<= 1) {  // value span 4 * lm
      const bool upper = (lane & lm) != 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], lm);
        v[i] = upper ? other - v[i] : v[i] + other;
      }
    }
    const float sc = 0.08838834764831845f;  // 128^-1/2
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = bf16_round(v[i] * sc);  // the transform returns bf16
  }
  if (fp4) {
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 6.f * 1.17549435e-38f);  // 6 * 2^-126
    // 2^ceil(log2(amax * (1/6))) from the exponent bits (kernel.py:22-37; the
    // reference multiplies by the fp32 reciprocal of 6)
    const uint32_t bits = __float_as_uint(__fmul_rn(amax, 1.f / 6.f));
    const int e = (int)((bits >> 23) & 0xff) - 127 + ((bits & 0x7fffffu) != 0 ? 1 : 0);
    const float s = __uint_as_float((uint32_t)(e + 127) << 23);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float q = fminf(fmaxf(__fdiv_rn(v[i], s), -6.f), 6.f);
      v[i] = bf16_round(__fmul_rn(e2m1_round(q), s));
    }
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
  reinterpret_cast<uint2*>(x + r * 128)[lane] =
      make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// ---------------------------------------------------------------- top-k

constexpr int kTopkThreads = 1024;
constexpr int kMaxK = 2048;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // larger float -> larger key
}

// Inclusive sum of v over the CTA's threads (thread order); `scratch` holds
// 32 words and is free again after the call's final barrier.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) scratch[wid] = v;
  __syncthreads();
  if (wid == 0) {
    uint32_t w = lane < (int)(blockDim.x >> 5) ? scratch[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    scratch[lane] = w;
  }
  __syncthreads();
  if (wid > 0) v += scratch[wid - 1];
  __syncthreads();
  return v;
}

// One CTA per row of `score` [rows, row_len]: out[row, :k] = the indices of
// the k largest scores, by score descending and, among equal scores, index
// ascending, plus `offset`; -inf scores, and with mask_ratio > 0 positions
// >= (row % s_len + 1) / mask_ratio, are never taken, so a row with fewer
// candidates than k ends in -1.  Radix select of the k-th largest key
// (digits of 11, 11 and 10 bits), the keys above it, the lowest-index keys
// equal to it (a CTA-wide scan in index order), then a bitonic sort.
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const float* __restrict__ score,
                                                            int64_t row_len, int k,
                                                            int32_t* __restrict__ out,
                                                            int64_t offset, int64_t s_len,
                                                            int mask_ratio) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t sel_key[kMaxK];
  __shared__ int32_t sel_idx[kMaxK];
  __shared__ uint32_t scratch[32];
  __shared__ uint32_t s_prefix, s_want, s_nout, s_nfin;
  const int64_t row = blockIdx.x;
  const float* sr = score + row * row_len;
  const int tid = threadIdx.x;
  // the prefill mask (model.py:522-526): query s sees positions < (s + 1) / ratio
  int64_t t_len = row_len;
  if (mask_ratio > 0) {
    const int64_t lim = (row % s_len + 1) / mask_ratio;
    if (lim < t_len) t_len = lim;
  }
  for (int i = tid; i < 2048; i += kTopkThreads) hist[i] = 0;
  if (tid == 0) {
    s_prefix = 0;
    s_nout = 0;
    s_nfin = 0;
  }
  __syncthreads();
  uint32_t kk = 0, mask_hi = 0;
  for (int pass = 0; pass < 3; pass++) {
    const int sh = pass == 0 ? 21 : pass == 1 ? 10 : 0;
    const int nb = pass == 2 ? 1024 : 2048;
    if (pass > 0) {
      for (int i = tid; i < nb; i += kTopkThreads) hist[i] = 0;
      __syncthreads();
    }
    const uint32_t pref = s_prefix;
    uint32_t fin = 0;
    for (int64_t i = tid; i < t_len; i += kTopkThreads) {
      const float f = sr[i];
      if (f == -INFINITY) continue;
      const uint32_t key = order_key(f);
      fin++;
      if ((key & mask_hi) == pref) atomicAdd(&hist[(key >> sh) & (nb - 1)], 1u);
    }
    if (pass == 0) {
      if (fin) atomicAdd(&s_nfin, fin);
      __syncthreads();
      kk = s_nfin < (uint32_t)k ? s_nfin : (uint32_t)k;
      if (tid == 0) s_want = kk;
      if (kk == 0) break;  // uniform: every thread read the same s_nfin
    }
    __syncthreads();
    // the digit holding the want-th largest key: thread t scans bins
    // nb-1-t*per .. nb-per-t*per (descending), a CTA scan orders the threads
    const int per = nb / kTopkThreads;
    const int top = nb - 1 - tid * per;
    uint32_t mine = 0;
    for (int j = 0; j < per; j++) mine += hist[top - j];
    const uint32_t want = s_want;
    const uint32_t incl = block_scan(mine, scratch);
    const uint32_t excl = incl - mine;
    if (excl < want && incl >= want) {
      uint32_t cum = excl;
      for (int j = 0; j < per; j++) {
        const uint32_t hcount = hist[top - j];
        if (cum + hcount >= want) {
          s_prefix = pref | ((uint32_t)(top - j) << sh);
          s_want = want - cum;
          break;
        }
        cum += hcount;
      }
    }
    mask_hi |= (uint32_t)(nb - 1) << sh;
    __syncthreads();
  }
  if (kk > 0) {
    const uint32_t kth = s_prefix, ties = s_want;  // keys equal to kth to take
    const uint32_t n_above = kk - ties;
    for (int64_t i = tid; i < t_len; i += kTopkThreads) {
      const float f = sr[i];
      if (f == -INFINITY) continue;
      const uint32_t key = order_key(f);
      if (key > kth) {
        const uint32_t p = atomicAdd(&s_nout, 1u);
        if (p < n_above) {
          sel_key[p] = key;
          sel_idx[p] = (int32_t)i;
        }
      }
    }
    // ties in index order: thread t owns the t-th contiguous chunk of the row
    const int64_t chunk = (t_len + kTopkThreads - 1) / kTopkThreads;
    const int64_t c0 = (int64_t)tid * chunk;
    const int64_t c1 = c0 + chunk < t_len ? c0 + chunk : t_len;
    uint32_t nt = 0;
    for (int64_t i = c0; i < c1; i++) nt += (sr[i] != -INFINITY && order_key(sr[i]) == kth) ? 1u : 0u;
    uint32_t r = block_scan(nt, scratch) - nt;
    for (int64_t i = c0; i < c1 && r < ties; i++) {
      if (sr[i] != -INFINITY && order_key(sr[i]) == kth) {
        sel_key[n_above + r] = kth;
        sel_idx[n_above + r] = (int32_t)i;
        r++;
      }
    }
    __syncthreads();
    // bitonic sort of the selection, padded to a power of two, by key
    // descending then index ascending
    int n2 = 1;
    while (n2 < (int)kk) n2 <<= 1;
    for (int i = (int)kk + tid; i < n2; i += kTopkThreads) {
      sel_key[i] = 0u;
      sel_idx[i] = 0x7fffffff;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < n2; i += kTopkThreads) {
          const int j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const uint32_t ki = sel_key[i], kj = sel_key[j];
            const int32_t ii = sel_idx[i], ij = sel_idx[j];
            const bool i_first = ki > kj || (ki == kj && ii < ij);
            if (i_first != desc) {
              sel_key[i] = kj;
              sel_key[j] = ki;
              sel_idx[i] = ij;
              sel_idx[j] = ii;
            }
          }
        }
        __syncthreads();
      }
    }
  }
  for (int i = tid; i < k; i += kTopkThreads)
    out[row * k + i] = i < (int)kk ? (int32_t)(sel_idx[i] + offset) : -1;
}

// ---------------------------------------------------------------- index lists

// window part (model.py:326-357) of row (b, s): width min(seqlen, window) at
// prefill, `window` at decode; the compress part (model.py:359-376, or the
// indexer's selection when `sel` is given) follows.
__global__ void index_lists_kernel(int32_t* __restrict__ out, int64_t bsz, int64_t seqlen,
                                   int64_t start_pos, int window, int ratio, int64_t offset,
                                   int win_w, int comp_w, const int32_t* __restrict__ sel) {
  const int64_t width = win_w + comp_w;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= bsz * seqlen * width) return;
  const int64_t j = i % width;
  const int64_t rs = i / width;  // (b, s)
  const int64_t s = rs % seqlen;
  int64_t v;
  if (j < win_w) {
    if (start_pos >= window - 1) {
      const int64_t sp = start_pos % window;
      v = j < window - sp - 1 ? sp + 1 + j : j - (window - sp - 1);
    } else if (start_pos > 0) {
      v = j <= start_pos ? j : -1;
    } else {
      const int64_t base = s - window + 1 > 0 ? s - window + 1 : 0;
      v = base + j;
      if (v > s) v = -1;
    }
  } else {
    const int64_t c = j - win_w;
    if (sel) {
      v = sel[rs * comp_w + c];  // the indexer's selection, offset already added
    } else if (start_pos > 0) {
      v = c + offset;  // arange((start_pos + 1) // ratio) + offset
    } else {
      v = c >= (s + 1) / ratio ? -1 : c + offset;
    }
  }
  out[i] = (int32_t)v;
}

}  // namespace

cudaError_t launch_rotate_fp4(void* x, int64_t rows, int hadamard, int fp4, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  rotate_fp4_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
      reinterpret_cast<__nv_bfloat16*>(x), rows, hadamard, fp4);
  return cudaGetLastError();
}

cudaError_t launch_topk(const float* score, int64_t rows, int64_t t_len, int k, int32_t* out,
                        int64_t offset, int64_t s_len, int mask_ratio, cudaStream_t st) {
  if (rows == 0 || k == 0) return cudaSuccess;
  if (k > kMaxK || (mask_ratio > 0 && s_len <= 0)) return cudaErrorInvalidValue;
  topk_kernel<<<(unsigned)rows, kTopkThreads, 0, st>>>(score, t_len, k, out, offset, s_len,
                                                       mask_ratio);
  return cudaGetLastError();
}

cudaError_t launch_index_lists(int32_t* out, int64_t bsz, int64_t seqlen, int64_t start_pos,
                               int window, int ratio, int64_t offset, int win_w, int comp_w,
                               const int32_t* sel, cudaStream_t st) {
  const int64_t n = bsz * seqlen * (win_w + comp_w);
  if (n == 0) return cudaSuccess;
  index_lists_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(out, bsz, seqlen, start_pos,
                                                                  window, ratio, offset, win_w,
                                                                  comp_w, sel);
  return cudaGetLastError();
}

}  // namespace qcau
