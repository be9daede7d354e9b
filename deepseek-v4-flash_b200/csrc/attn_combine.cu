// attn_combine.cu -- merge of split-KV attention partials, and the bounded
// flag wait of the peer-memory partial exchange.
//
// A query row's KV range, split over CTAs (split-KV) or over ranks (context
// parallel), leaves per split the partial softmax state (running max m_i in
// log2 units, denominator l_i, and O_i relative to m_i); the merge is the
// reference's online softmax applied across splits
// (Deepseek_origin/inference/kernel.py:331-348): M = max m_i,
// L = sum l_i 2^(m_i - M) + the sink term (added once, kernel.py:345-346),
// O = sum O_i 2^(m_i - M) / L, then the optional inverse RoPE of the V4 output
// (QCAU/QCAU_inference/inference/QCAU.py:313-319) and bf16 rounding.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// Inverse RoPE of one (re, im) pair of a bf16 output row (QCAU.py:313-319):
// the reference rotates the bf16 attention output, so round first.
__device__ __forceinline__ void inv_rope_pair(float& x, float& y, float2 cs) {
  x = bf16_round(x);
  y = bf16_round(y);
  const float re = __fadd_rn(__fmul_rn(x, cs.x), __fmul_rn(y, cs.y));
  const float im = __fsub_rn(__fmul_rn(y, cs.x), __fmul_rn(x, cs.y));
  x = re;
  y = im;
}

// Merge split-KV partials: M = max m_i, L = sum l_i 2^(m_i-M) + sink term,
// O = sum acc_i 2^(m_i-M) / L.  One warp per (query, head).  Partials are
// [rows][splits][h], or [splits][rows][h] with part_split_major (the ranks'
// blocks of a context-parallel decode, after their exchange).
__global__ void attn_combine_kernel(AttnArgs p) {
  const int lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = p.b * p.s;
  if (task >= rows * p.h) return;
  const int64_t qrow = task / p.h, hh = task % p.h;
  const int64_t tpos = qrow % p.s;
  const int64_t prow0 = p.part_split_major ? qrow * p.h + hh : qrow * p.splits * p.h + hh;
  const int64_t pstride = p.part_split_major ? rows * p.h : p.h;  // between splits, in rows
  const float* ml = p.part_ml + prow0 * 2;
  const int64_t ml_stride = pstride * 2;
  float M = -INFINITY;
  for (int i = 0; i < p.splits; i++) M = fmaxf(M, ml[i * ml_stride]);
  float L = 0.f;
  for (int i = 0; i < p.splits; i++) {
    const float mi = ml[i * ml_stride];
    if (mi != -INFINITY) L += ml[i * ml_stride + 1] * exp2f(mi - M);
  }
  const float sk = p.sink ? p.sink[hh] * kLog2e : -INFINITY;
  if (M != -INFINITY)
    L += exp2f(sk - M);
  else
    L += (p.sink && isfinite(p.sink[hh])) ? 1.f : 0.f;
  const float inv = 1.f / fmaxf(L, 1.17549435e-38f);
  const int64_t ob = p.o_hblock > 0 ? p.o_hblock : p.h;  // o in head blocks of ob
  const int64_t oblk = hh / ob;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.o) +
                       ((oblk * rows + qrow) * ob + (hh - oblk * ob)) * p.d_v;
  const int64_t po0 = prow0 * p.d_v;
  const int64_t po_stride = pstride * p.d_v;
  for (int c = lane * 4; c < p.d_v; c += 128) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < p.splits; i++) {
      const float mi = ml[i * ml_stride];
      if (mi == -INFINITY) continue;
      const int64_t e = po0 + i * po_stride + c;
      float4 v;
      float w = exp2f(mi - M);
      if (p.part_f16) {  // O / l: weighted by l
        const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.part_o) + e);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        v = make_float4(lo.x, lo.y, hi.x, hi.y);
        w *= ml[i * ml_stride + 1];
      } else {
        v = *reinterpret_cast<const float4*>(p.part_o + e);
      }
      a.x = fmaf(v.x, w, a.x);
      a.y = fmaf(v.y, w, a.y);
      a.z = fmaf(v.z, w, a.z);
      a.w = fmaf(v.w, w, a.w);
    }
    a.x *= inv;
    a.y *= inv;
    a.z *= inv;
    a.w *= inv;
    if (p.inv_rope && c >= p.d_v - p.rope_dim) {
      const float2* f = reinterpret_cast<const float2*>(p.freqs) +
                        (p.pos0 + tpos) * (p.rope_dim / 2) + (c - (p.d_v - p.rope_dim)) / 2;
      inv_rope_pair(a.x, a.y, f[0]);
      inv_rope_pair(a.z, a.w, f[1]);
    }
    *reinterpret_cast<__nv_bfloat162*>(out + c) = __floats2bfloat162_rn(a.x, a.y);
    *reinterpret_cast<__nv_bfloat162*>(out + c + 2) = __floats2bfloat162_rn(a.z, a.w);
  }
}

// The same merge for 512-wide outputs (the latent width), with the loads of
// a split issued together: lane l holds dims 4l + 128k (k < 4), each
// split's weight is computed once, and all four loads of a split precede its
// arithmetic (four splits in flight).  An empty split (max -inf, its O never
// written) is not loaded (the predicate is the same for the whole warp) and
// adds zeros, so stale values never enter the sums.  The arithmetic and its
// order are attn_combine_kernel's.
template <bool kF16>
__global__ void __launch_bounds__(256) attn_combine512_kernel(AttnArgs p) {
  const int lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = p.b * p.s;
  if (task >= rows * p.h) return;
  const int64_t qrow = task / p.h, hh = task % p.h;
  const int64_t tpos = qrow % p.s;
  const int64_t prow0 = p.part_split_major ? qrow * p.h + hh : qrow * p.splits * p.h + hh;
  const int64_t pstride = p.part_split_major ? rows * p.h : p.h;  // between splits, in rows
  const float* ml = p.part_ml + prow0 * 2;
  const int64_t ml_stride = pstride * 2;
  const int ns = p.splits;
  // Up to 32 splits: lane i loads (m_i, l_i) of split i, so the warp's
  // softmax states arrive in one round trip and are read back by shuffles in
  // split order (the sums below are the same, term for term).
  const bool lanes = ns <= 32;
  float2 mine = make_float2(-INFINITY, 0.f);
  if (lanes && lane < ns) mine = *reinterpret_cast<const float2*>(ml + lane * ml_stride);
  auto m_of = [&](int i) {
    return lanes ? __shfl_sync(0xffffffffu, mine.x, i) : ml[i * ml_stride];
  };
  auto l_of = [&](int i) {
    return lanes ? __shfl_sync(0xffffffffu, mine.y, i) : ml[i * ml_stride + 1];
  };
  float M = -INFINITY;
  for (int i = 0; i < ns; i++) M = fmaxf(M, m_of(i));
  float L = 0.f;
  for (int i = 0; i < ns; i++) {
    const float mi = m_of(i), li = l_of(i);
    if (mi != -INFINITY) L += li * exp2f(mi - M);
  }
  const float sk = p.sink ? p.sink[hh] * kLog2e : -INFINITY;
  if (M != -INFINITY)
    L += exp2f(sk - M);
  else
    L += (p.sink && isfinite(p.sink[hh])) ? 1.f : 0.f;
  const float inv = 1.f / fmaxf(L, 1.17549435e-38f);

  float a[16];
#pragma unroll
  for (int j = 0; j < 16; j++) a[j] = 0.f;
  const int64_t base = prow0 * 512 + lane * 4;
  const int64_t po_stride = pstride * 512;
#pragma unroll 4
  for (int i = 0; i < ns; i++) {
    const float mi = m_of(i), li = l_of(i);
    const bool live = mi != -INFINITY;
    const int64_t e = base + i * po_stride;
    float v[16];
    float w;
    if constexpr (kF16) {  // O / l: weighted by l
      const __half* src = reinterpret_cast<const __half*>(p.part_o) + e;
      uint2 u[4];
#pragma unroll
      for (int k = 0; k < 4; k++)
        u[k] = live ? *reinterpret_cast<const uint2*>(src + 128 * k) : make_uint2(0u, 0u);
      w = live ? exp2f(mi - M) * li : 0.f;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u[k].x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u[k].y));
        v[4 * k] = lo.x;
        v[4 * k + 1] = lo.y;
        v[4 * k + 2] = hi.x;
        v[4 * k + 3] = hi.y;
      }
    } else {
      const float* src = p.part_o + e;
      float4 f[4];
#pragma unroll
      for (int k = 0; k < 4; k++)
        f[k] = live ? *reinterpret_cast<const float4*>(src + 128 * k) : make_float4(0.f, 0.f, 0.f, 0.f);
      w = live ? exp2f(mi - M) : 0.f;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        v[4 * k] = f[k].x;
        v[4 * k + 1] = f[k].y;
        v[4 * k + 2] = f[k].z;
        v[4 * k + 3] = f[k].w;
      }
    }
#pragma unroll
    for (int j = 0; j < 16; j++) a[j] = fmaf(live ? v[j] : 0.f, w, a[j]);
  }

  const int64_t ob = p.o_hblock > 0 ? p.o_hblock : p.h;  // o in head blocks of ob
  const int64_t oblk = hh / ob;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.o) +
                       ((oblk * rows + qrow) * ob + (hh - oblk * ob)) * 512;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const int c = lane * 4 + 128 * k;
    float x0 = a[4 * k] * inv, x1 = a[4 * k + 1] * inv;
    float x2 = a[4 * k + 2] * inv, x3 = a[4 * k + 3] * inv;
    if (p.inv_rope && c >= 512 - p.rope_dim) {
      const float2* f = reinterpret_cast<const float2*>(p.freqs) +
                        (p.pos0 + tpos) * (p.rope_dim / 2) + (c - (512 - p.rope_dim)) / 2;
      inv_rope_pair(x0, x1, f[0]);
      inv_rope_pair(x2, x3, f[1]);
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(x0, x1), hi = __floats2bfloat162_rn(x2, x3);
    *reinterpret_cast<uint2*>(out + c) =
        make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  }
}

}  // namespace

// One thread per flag: spin (bounded) until flags[i] >= epoch, acquiring at
// system scope what the peer that raised it wrote before its release.
__global__ void wait_flags_kernel(const uint32_t* flags, int n, uint32_t epoch, int* err) {
  const int i = threadIdx.x;
  if (i >= n) return;
  const long long t0 = clock64();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if (clock64() - t0 > kWaitLimitCycles) {
      raise_dev_error(err, QCAU_DEVERR_TIMEOUT);
      break;
    }
    __nanosleep(64);
  }
}

cudaError_t launch_wait_flags(const uint32_t* flags, int n, uint32_t epoch, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (n > 1024) return cudaErrorInvalidValue;
  wait_flags_kernel<<<1, ((n + 31) / 32) * 32, 0, st>>>(flags, n, epoch, device_error_word());
  return cudaGetLastError();
}

cudaError_t launch_attn_combine(const AttnArgs& p, cudaStream_t st) {
  const int64_t tasks = p.b * p.s * p.h;
  if (tasks == 0) return cudaSuccess;
  if (p.d_v % 128) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((tasks + 7) / 8);
  if (p.d_v == 512 && p.part_f16)
    attn_combine512_kernel<true><<<grid, 256, 0, st>>>(p);
  else if (p.d_v == 512)
    attn_combine512_kernel<false><<<grid, 256, 0, st>>>(p);
  else
    attn_combine_kernel<<<grid, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace qcau
