// attn_general.cu -- split-KV MQA attention over gathered or paged latent rows.
//
// Semantics follow the reference attention core
// (Deepseek_origin/inference/kernel.py:276-352, with the guards of
// QCAU/QCAU_inference/inference/QCAU.py:176-242):
//   * keys come in tiles of 64 (kernel.py:290); an index outside [0, n_kv)
//     (the reference's -1) gives a -inf score and a zero row (:322-327);
//   * online softmax with a running fp32 max; a tile with no valid key leaves
//     the running max unchanged (QCAU.py:201-216);
//   * P is rounded to bf16 before P.V while the denominator sums fp32 P
//     (kernel.py:337-343);
//   * the attention sink enters the denominator once, after the loop
//     (kernel.py:345-346); no valid key at all -> output 0 (QCAU.py guard).
// K rows are kv[..., :d_qk] and V rows kv[..., :d_v] of the same latent row
// (V4: one 512-wide row; absorbed MLA: 576-wide row, V = first 512).
//
// CTA = 16 query heads of one query token x one KV split, 8 warps:
//   S = Q K^T : warp w computes keys [8w, 8w+8) of the tile (mma.sync m16n8k16)
//   softmax   : row max reduced across warps through shared memory
//   O += P V  : warp w owns output dims [w*d_v/8, (w+1)*d_v/8)
// Rows are fetched with 16-byte cp.async into a double-buffered tile.
// With one split the epilogue writes bf16 output (optionally inverse RoPE);
// with several it writes fp32 partials (acc, max, sum) for attn_combine.
// Scores are kept in log2 units (scale * log2 e folded in) so exp2 is used.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kTileKeys = 64;
constexpr int kHeadsPerCta = 16;
constexpr int kWarps = 8;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                        uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Eight e4m3 codes times a row scale, as eight bf16 (e4m3 -> f16 is exact).
__device__ __forceinline__ uint4 e4m3x8_scaled_bf16(uint2 raw, float s) {
  uint32_t out[4];
  const uint32_t w[2] = {raw.x, raw.y};
#pragma unroll
  for (int k = 0; k < 2; k++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint16_t two = (uint16_t)(w[k] >> (16 * h));
      uint32_t f16x2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(f16x2) : "h"(two));
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&f16x2));
      __nv_bfloat162 b = __floats2bfloat162_rn(f.x * s, f.y * s);
      out[2 * k + h] = *reinterpret_cast<uint32_t*>(&b);
    }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

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

template <int DQK, int DV>
struct Cfg {
  static constexpr int kRow = DQK + 8;  // padded smem row (elements)
  static constexpr int kQBytes = kHeadsPerCta * kRow * 2;
  static constexpr int kKvBytes = kTileKeys * kRow * 2;
  static constexpr int kPRow = kTileKeys + 8;
  static constexpr int kPBytes = kHeadsPerCta * kPRow * 2;
  static constexpr int kNPerWarp = DV / kWarps;  // output dims per warp
  static constexpr int kNTiles = kNPerWarp / 8;
  static constexpr size_t kSmem = kQBytes + 2 * kKvBytes + kPBytes + 2 * kTileKeys * 4 +
                                  2 * kWarps * kHeadsPerCta * 4 + 64;
  static_assert(DQK % 16 == 0 && DV % 64 == 0 && DV <= DQK, "unsupported widths");
};

template <int DQK, int DV>
__global__ void __launch_bounds__(kWarps * 32, 1) attn_general_kernel(AttnArgs p, int* err) {
  using C = Cfg<DQK, DV>;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sKV = reinterpret_cast<__nv_bfloat16*>(smem + C::kQBytes);
  __nv_bfloat16* sP = reinterpret_cast<__nv_bfloat16*>(smem + C::kQBytes + 2 * C::kKvBytes);
  int* sValid = reinterpret_cast<int*>(smem + C::kQBytes + 2 * C::kKvBytes + C::kPBytes);
  float* sMax = reinterpret_cast<float*>(sValid + 2 * kTileKeys);  // [warps][16]
  float* sSum = sMax + kWarps * kHeadsPerCta;                       // [warps][16]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t qrow = blockIdx.x;  // query token index in [0, b*s)
  const int h0 = blockIdx.y * kHeadsPerCta;
  const int split = blockIdx.z;
  const int64_t bidx = qrow / p.s, tpos = qrow % p.s;
  const bool paged = p.block_table != nullptr;

  // key list length and this split's tile range
  // paged: query t of s sees the cached prefix up to its own position
  const int64_t len = paged ? (int64_t)p.seqlens[bidx] - (p.s - 1 - tpos) : p.topk;
  const int64_t ntiles = (len + kTileKeys - 1) / kTileKeys;
  const int64_t t_begin = ntiles * split / p.splits;
  const int64_t t_end = ntiles * (split + 1) / p.splits;

  // ---- Q tile (rows beyond h are zero)
  {
    constexpr int kChunks = DQK / 8;
    for (int i = tid; i < kHeadsPerCta * kChunks; i += kWarps * 32) {
      const int r = i / kChunks, c = i % kChunks;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h0 + r < p.h)
        v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.q) +
                                            (qrow * p.h + h0 + r) * p.q_row_stride + c * 8);
      *reinterpret_cast<uint4*>(sQ + r * C::kRow + c * 8) = v;
    }
  }

  auto load_tile = [&](int64_t t, int buf) {
    __nv_bfloat16* dst = sKV + (size_t)buf * kTileKeys * C::kRow;
    int* vld = sValid + buf * kTileKeys;
    constexpr int kChunks = DQK / 8;
    for (int i = tid; i < kTileKeys * kChunks; i += kWarps * 32) {
      const int r = i / kChunks, c = i % kChunks;
      const int64_t j = t * kTileKeys + r;
      const __nv_bfloat16* src = nullptr;
      if (j < len) {
        if (paged) {
          const int64_t page = p.block_table[bidx * p.max_pages + j / p.page_size];
          if (page >= 0 && page < p.num_pages)
            src = reinterpret_cast<const __nv_bfloat16*>(p.kv) +
                  (page * p.page_size + j % p.page_size) * p.d_kv;
          else if (c == 0)
            raise_dev_error(err, QCAU_DEVERR_INDEX);
        } else {
          const int64_t id = p.idx[qrow * p.topk + j];
          if (id >= 0 && id < p.n_kv)
            src = reinterpret_cast<const __nv_bfloat16*>(p.kv) + (bidx * p.n_kv + id) * p.d_kv;
        }
      }
      if (c == 0) vld[r] = src != nullptr;
      const uint32_t d = smem_u32(dst + r * C::kRow + c * 8);
      if (src)
        cp_async16(d, src + c * 8);
      else
        *reinterpret_cast<uint4*>(dst + r * C::kRow + c * 8) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };

  // FP8 latent rows (gather mode): the e4m3 codes of tile t+1 are loaded
  // into registers before tile t is computed and converted to bf16 after it,
  // so the gather latency overlaps the math; the rope part goes by cp.async
  const bool fp8 = DQK == 576 && p.kv_fp8 != nullptr;  // 576 = 512 codes + 64 rope
  constexpr int kFp8Chunks = kTileKeys * 64 / (kWarps * 32);  // 8-code chunks per thread
  uint2 fraw[kFp8Chunks];
  float fsc[kFp8Chunks];
  auto fp8_row = [&](int64_t t, int r) -> int64_t {
    const int64_t j = t * kTileKeys + r;
    if (j >= len) return -1;
    const int64_t id = p.idx[qrow * p.topk + j];
    return (id >= 0 && id < p.n_kv) ? bidx * p.n_kv + id : -1;
  };
  auto issue_fp8 = [&](int64_t t, int buf) {
    __nv_bfloat16* dst = sKV + (size_t)buf * kTileKeys * C::kRow;
    int* vld = sValid + buf * kTileKeys;
#pragma unroll
    for (int k = 0; k < kFp8Chunks; k++) {
      const int i = tid + k * kWarps * 32, r = i >> 6, c = i & 63;
      const int64_t row = fp8_row(t, r);
      if (c == 0) vld[r] = row >= 0;
      if (row >= 0) {
        fraw[k] = __ldg(reinterpret_cast<const uint2*>(p.kv_fp8 + row * 512 + c * 8));
        fsc[k] = __ldg(p.kv_scale + row);
      } else {
        fraw[k] = make_uint2(0u, 0u);
        fsc[k] = 0.f;
      }
    }
    for (int i = tid; i < kTileKeys * 8; i += kWarps * 32) {
      const int r = i >> 3, c = i & 7;
      const int64_t row = fp8_row(t, r);
      const uint32_t d = smem_u32(dst + r * C::kRow + 512 + c * 8);
      if (row >= 0)
        cp_async16(d, reinterpret_cast<const __nv_bfloat16*>(p.kv_rope) + row * 64 + c * 8);
      else
        *reinterpret_cast<uint4*>(dst + r * C::kRow + 512 + c * 8) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };
  auto finish_fp8 = [&](int buf) {
    __nv_bfloat16* dst = sKV + (size_t)buf * kTileKeys * C::kRow;
#pragma unroll
    for (int k = 0; k < kFp8Chunks; k++) {
      const int i = tid + k * kWarps * 32, r = i >> 6, c = i & 63;
      *reinterpret_cast<uint4*>(dst + r * C::kRow + c * 8) = e4m3x8_scaled_bf16(fraw[k], fsc[k]);
    }
  };

  // running state: this thread's two rows (lane/4 and lane/4 + 8)
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_part[2] = {0.f, 0.f};  // this warp's share of the denominator
  float acc[C::kNTiles][4];
#pragma unroll
  for (int i = 0; i < C::kNTiles; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const float sl2 = p.scale * kLog2e;
  const int r0 = lane >> 2, cq = (lane & 3) * 2;

  if (t_begin < t_end) {
    if (fp8) {
      issue_fp8(t_begin, 0);
      finish_fp8(0);
    } else {
      load_tile(t_begin, 0);
    }
  }
  for (int64_t t = t_begin; t < t_end; t++) {
    const int buf = (int)((t - t_begin) & 1);
    if (t + 1 < t_end) {
      if (fp8)
        issue_fp8(t + 1, buf ^ 1);
      else
        load_tile(t + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* kv = sKV + (size_t)buf * kTileKeys * C::kRow;
    const int* vld = sValid + buf * kTileKeys;

    // ---- S = Q K^T for keys [8w, 8w+8)
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const uint32_t qa = smem_u32(sQ + (lane & 15) * C::kRow + (lane >> 4) * 8);
      const uint32_t kb = smem_u32(kv + (warp * 8 + (lane & 7)) * C::kRow + ((lane >> 3) & 1) * 8);
#pragma unroll 4
      for (int k0 = 0; k0 < DQK; k0 += 16) {
        uint32_t a0, a1, a2, a3, b0, b1;
        ldsm_x4(a0, a1, a2, a3, qa + k0 * 2);
        ldsm_x2(b0, b1, kb + k0 * 2);
        mma16816(s, a0, a1, a2, a3, b0, b1);
      }
    }
    const bool v0 = vld[warp * 8 + cq] != 0, v1 = vld[warp * 8 + cq + 1] != 0;
    s[0] = v0 ? s[0] * sl2 : -INFINITY;
    s[1] = v1 ? s[1] * sl2 : -INFINITY;
    s[2] = v0 ? s[2] * sl2 : -INFINITY;
    s[3] = v1 ? s[3] * sl2 : -INFINITY;
    float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    if ((lane & 3) == 0) {
      sMax[warp * kHeadsPerCta + r0] = mx0;
      sMax[warp * kHeadsPerCta + r0 + 8] = mx1;
    }
    __syncthreads();
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; w++) {
      tmax0 = fmaxf(tmax0, sMax[w * kHeadsPerCta + r0]);
      tmax1 = fmaxf(tmax1, sMax[w * kHeadsPerCta + r0 + 8]);
    }
    // a tile without any valid key leaves the state untouched
    const float mn0 = fmaxf(m_run[0], tmax0), mn1 = fmaxf(m_run[1], tmax1);
    const float al0 = (tmax0 == -INFINITY) ? 1.f : exp2f(m_run[0] - mn0);
    const float al1 = (tmax1 == -INFINITY) ? 1.f : exp2f(m_run[1] - mn1);
    const float p0 = v0 ? exp2f(s[0] - mn0) : 0.f;
    const float p1 = v1 ? exp2f(s[1] - mn0) : 0.f;
    const float p2 = v0 ? exp2f(s[2] - mn1) : 0.f;
    const float p3 = v1 ? exp2f(s[3] - mn1) : 0.f;
    m_run[0] = (tmax0 == -INFINITY) ? m_run[0] : mn0;
    m_run[1] = (tmax1 == -INFINITY) ? m_run[1] : mn1;
    l_part[0] = l_part[0] * al0 + (p0 + p1);
    l_part[1] = l_part[1] * al1 + (p2 + p3);
    *reinterpret_cast<__nv_bfloat162*>(sP + r0 * C::kPRow + warp * 8 + cq) =
        __floats2bfloat162_rn(p0, p1);
    *reinterpret_cast<__nv_bfloat162*>(sP + (r0 + 8) * C::kPRow + warp * 8 + cq) =
        __floats2bfloat162_rn(p2, p3);
#pragma unroll
    for (int i = 0; i < C::kNTiles; i++) {
      acc[i][0] *= al0;
      acc[i][1] *= al0;
      acc[i][2] *= al1;
      acc[i][3] *= al1;
    }
    __syncthreads();
    // ---- O += P V for dims [warp*kNPerWarp, ...)
    {
      const uint32_t pa = smem_u32(sP + (lane & 15) * C::kPRow + (lane >> 4) * 8);
#pragma unroll
      for (int k0 = 0; k0 < kTileKeys; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a0, a1, a2, a3, pa + k0 * 2);
        const uint32_t vb = smem_u32(kv + (k0 + (lane & 15)) * C::kRow + warp * C::kNPerWarp);
#pragma unroll
        for (int i = 0; i < C::kNTiles; i++) {
          uint32_t b0, b1;
          ldsm_x2_t(b0, b1, vb + i * 16);
          mma16816(acc[i], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    if (fp8 && t + 1 < t_end) finish_fp8(buf ^ 1);
    __syncthreads();  // sP and the KV buffer are rewritten next iteration
  }

  // ---- denominator: the 4 lanes of a row, then the 8 warps
  float lp0 = l_part[0], lp1 = l_part[1];
  lp0 += __shfl_xor_sync(0xffffffffu, lp0, 1);
  lp0 += __shfl_xor_sync(0xffffffffu, lp0, 2);
  lp1 += __shfl_xor_sync(0xffffffffu, lp1, 1);
  lp1 += __shfl_xor_sync(0xffffffffu, lp1, 2);
  if ((lane & 3) == 0) {
    sSum[warp * kHeadsPerCta + r0] = lp0;
    sSum[warp * kHeadsPerCta + r0 + 8] = lp1;
  }
  __syncthreads();
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; w++) {
    l0 += sSum[w * kHeadsPerCta + r0];
    l1 += sSum[w * kHeadsPerCta + r0 + 8];
  }
  const int ha = h0 + r0, hb = h0 + r0 + 8;
  const int ncol0 = warp * C::kNPerWarp;

  if (p.splits > 1) {
    // fp32 partials for attn_combine: acc relative to m (log2 units), (m, l)
    for (int half = 0; half < 2; half++) {
      const int hh = half ? hb : ha;
      if (hh >= p.h) continue;
      const int64_t prow = (qrow * p.splits + split) * p.h + hh;
      float* po = p.part_o + prow * DV;
#pragma unroll
      for (int i = 0; i < C::kNTiles; i++)
        *reinterpret_cast<float2*>(po + ncol0 + i * 8 + cq) =
            make_float2(acc[i][half * 2], acc[i][half * 2 + 1]);
      if (warp == 0 && (lane & 3) == 0) {
        p.part_ml[prow * 2] = half ? m_run[1] : m_run[0];
        p.part_ml[prow * 2 + 1] = half ? l1 : l0;
      }
    }
    return;
  }

  // ---- single split: normalise, sink, optional inverse RoPE, bf16 store
  for (int half = 0; half < 2; half++) {
    const int hh = half ? hb : ha;
    if (hh >= p.h) continue;
    const float m = half ? m_run[1] : m_run[0];
    const float l = half ? l1 : l0;
    const float sk = p.sink ? p.sink[hh] * kLog2e : -INFINITY;
    float term;
    if (m != -INFINITY)
      term = exp2f(sk - m);
    else
      term = (p.sink && isfinite(p.sink[hh])) ? 1.f : 0.f;
    const float inv = 1.f / fmaxf(l + term, 1.17549435e-38f);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.o) + (qrow * p.h + hh) * DV;
#pragma unroll
    for (int i = 0; i < C::kNTiles; i++) {
      const int col = ncol0 + i * 8 + cq;
      float x = acc[i][half * 2] * inv, y = acc[i][half * 2 + 1] * inv;
      if (p.inv_rope && col >= DV - p.rope_dim)
        inv_rope_pair(x, y, reinterpret_cast<const float2*>(p.freqs)[(p.pos0 + tpos) * (p.rope_dim / 2) +
                                                                   (col - (DV - p.rope_dim)) / 2]);
      *reinterpret_cast<__nv_bfloat162*>(out + col) = __floats2bfloat162_rn(x, y);
    }
  }
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
// arithmetic (two splits in flight).  An empty split (max -inf, its O never
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

  float a[16];
#pragma unroll
  for (int j = 0; j < 16; j++) a[j] = 0.f;
  const int64_t base = prow0 * 512 + lane * 4;
  const int64_t po_stride = pstride * 512;
#pragma unroll 2
  for (int i = 0; i < p.splits; i++) {
    const float mi = ml[i * ml_stride];
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
      w = live ? exp2f(mi - M) * ml[i * ml_stride + 1] : 0.f;
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

template <int DQK, int DV>
cudaError_t launch_t(const AttnArgs& p, cudaStream_t st) {
  using C = Cfg<DQK, DV>;
  cudaError_t e = cudaFuncSetAttribute(attn_general_kernel<DQK, DV>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(p.b * p.s), (unsigned)((p.h + kHeadsPerCta - 1) / kHeadsPerCta),
            (unsigned)p.splits);
  attn_general_kernel<DQK, DV><<<grid, kWarps * 32, C::kSmem, st>>>(p, device_error_word());
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attn_general(const AttnArgs& p, cudaStream_t st) {
  if (p.b * p.s == 0 || p.h == 0) return cudaSuccess;
  if (p.d_qk == 576 && p.d_v == 512) return launch_t<576, 512>(p, st);
  if (p.d_qk == 512 && p.d_v == 512) return launch_t<512, 512>(p, st);
  return cudaErrorNotSupported;
}

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
