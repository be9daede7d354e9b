// attn_gather_sm100.cu -- tcgen05 split-KV attention over gathered latent rows.
//
// The key list of a query row is either its top-k indices into the latent
// rows of its sequence (the reference's sparse attention,
// Deepseek_origin/inference/kernel.py:276-352: an index outside [0, n_kv),
// the reference's -1, gives a -inf score and a zero row), or the first
// seqlen tokens of a paged cache (a decode or causal-prefill row).  The rows
// are bf16 [.., d_kv], or the FP8 latent format: e4m3 codes [.., 512] with one
// fp32 scale per row and a bf16 rope part [.., 64], whose value is
// bf16(e4m3 * scale) followed by the rope part.  K is the first d_qk values
// of a row (512 or 576) and V its first 512.
//
// Numerics are the reference's: fp32 scores, an exact running max per tile,
// P rounded to bf16 before P.V, the denominator summed from fp32 P, the sink
// added once after the loop (kernel.py:331-348), and no output for a row
// without any valid key (QCAU/QCAU_inference/inference/QCAU.py:201-242).
//
// One CTA = one query row x one group of NH heads (16, 32 or 64) x one KV
// split.  Every gathered row is loaded once per head group, and the heads are
// the N dimension of both MMAs, so a 16-head shard does not pad the tensor
// work to 64 or 128 rows:
//   QK : tcgen05 kind::f16, M = 64 gathered rows, N = NH heads, K = d_qk in
//        chunks of 64: S^T in TMEM (M = 64 layout: rows 16q..16q+15 in lanes
//        32q..32q+15), two buffers;
//   PV : M = 128 latent dims (4 MMAs cover 512), N = NH heads, K = 64 rows:
//        A = the same staged rows read MN-major (dims contiguous), B = P^T
//        (K-major [head][row]); O^T in TMEM, lanes = dims, one column a head.
// Rows are staged in 128-byte-swizzled 64-dim chunks [chunk][64 rows][128 B]
// (the UMMA K-major layout), two tile slots.  Two groups of four producer
// warps gather alternate tiles (group g fills slot g), so two tiles are in
// flight: bf16 rows by 16-byte cp.async, FP8 codes through registers (loaded
// before the slot is free, converted after).  Softmax: four warps read S^T
// (a thread per row), stage it in shared memory as [head][row], and then
// NH heads x (128 / NH) threads each reduce, exponentiate and write P^T; a
// tile that raises a head's max rescales that head's O^T column in TMEM.
// Warps: 0-3 softmax / epilogue, 4 QK issuer + TMEM allocator, 5 PV issuer,
// 6-9 and 10-13 the two producer groups.
// With one split the epilogue normalises, adds the sink, applies the
// optional inverse RoPE (V4 mode, QCAU.py:313-319) and writes bf16; with
// several it writes fp32 partials (O relative to its max, max in log2 units,
// sum) for attn_combine.
// Every wait is bounded; a timeout raises QCAU_DEVERR_TIMEOUT, lets the copies
// and MMAs in flight finish, frees TMEM and returns.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kTok = 64;        // gathered rows per tile
constexpr int kSoft = 128;      // softmax / epilogue threads (warps 0-3)
constexpr int kQkWarp = 4;
constexpr int kPvWarp = 5;
constexpr int kProd0 = 6;       // first producer warp
constexpr int kGroupWarps = 4;  // warps per producer group
constexpr int kThreads = (kProd0 + 2 * kGroupWarps) * 32;  // 448
constexpr float kLog2e = 1.4426950408889634f;

struct GatherShared {
  uint64_t kv_full[2];   // producer group g filled slot g (128 arrivals)
  uint64_t kv_empty[2];  // PV of the slot's tile done
  uint64_t q_full;       // Q staged (producer group 0)
  uint64_t s_full[2];    // QK done into S^T buffer b
  uint64_t s_free[2];    // the 4 softmax warps read S^T buffer b
  uint64_t p_full;       // P^T written and O^T rescaled (4 softmax warps)
  uint64_t p_free;       // PV done with P^T and O^T
  uint64_t o_full;       // last PV done
  uint64_t xa, xb, xc;   // softmax warps: S staged / alphas written / denominators written
  int valid[2][kTok];
  int resc[4];
  float alpha[64];
  float m_fin[64];
  float l_fin[64];
  uint32_t tmem_base;
  int abort;
};

template <int NH, int DQK>
struct GCfg {
  static constexpr int kChunks = DQK / 64;
  static constexpr int kQBytes = NH * DQK * 2;       // [chunk][NH rows][128 B]
  static constexpr int kSlotBytes = kChunks * 8192;  // [chunk][64 rows][128 B]
  static constexpr int kPBytes = NH * 128;           // P^T [NH rows][64 rows of the tile]
  static constexpr int kSBytes = NH * kTok * 4;      // S^T staged as [head][row] fp32
  static constexpr uint32_t kColO = 0;               // O^T: 4 blocks of NH columns
  static constexpr uint32_t kColS = 4 * NH;          // S^T: 2 buffers of NH columns
  static constexpr uint32_t kCols = 6 * NH <= 128 ? 128 : (6 * NH <= 256 ? 256 : 512);
  static constexpr int kTph = kSoft / NH;            // softmax threads per head
  static constexpr int kTpt = kTok / kTph;           // rows per softmax thread
  static constexpr size_t kSmem = 1024 + (size_t)kQBytes + 2 * (size_t)kSlotBytes + kPBytes +
                                  kSBytes + sizeof(GatherShared);
  static_assert(NH == 16 || NH == 32 || NH == 64, "heads per CTA");
  static_assert(DQK == 512 || DQK == 576, "key width");
  static_assert(kSmem <= 232448, "shared memory budget");
};

struct GatherParams {
  const __nv_bfloat16* q;
  int64_t q_row_stride;
  const __nv_bfloat16* kv;    // bf16 rows
  const uint8_t* kv_fp8;      // FP8 rows: codes, scales, rope part
  const float* kv_scale;
  const __nv_bfloat16* kv_rope;
  const int32_t* idx;         // gather mode
  const int32_t* table;       // paged mode
  const int32_t* seqlens;
  const float* sink;
  __nv_bfloat16* out;
  float* part_o;
  float* part_ml;
  const float* freqs;
  int* err;
  int64_t rows, s, h, n_kv, topk, d_kv, page_size, max_pages, num_pages, pos0;
  int hgroups, splits, inv_rope, rope_dim;
  float scale;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void st_shared16(uint32_t dst, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ int64_t shfl_i64(int64_t v, int src) {
  const int lo = __shfl_sync(0xffffffffu, (int)(uint32_t)(uint64_t)v, src);
  const int hi = __shfl_sync(0xffffffffu, (int)(uint32_t)((uint64_t)v >> 32), src);
  return (int64_t)(((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo);
}

// Eight e4m3 codes times the row scale as eight bf16: e4m3 -> f16 is exact,
// then fp32 multiply and round to bf16 (the value bf16(e4m3 * scale)).
__device__ __forceinline__ uint4 e4m3x8_to_bf16(uint32_t w0, uint32_t w1, float s) {
  uint32_t out[4];
  const uint32_t w[2] = {w0, w1};
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

// Inverse RoPE of one (re, im) pair of the bf16 attention output
// (QCAU.py:313-319): round to bf16 first, as the reference rotates its bf16
// output, then rotate by the conjugate in fp32.
__device__ __forceinline__ void inv_rope(float& x, float& y, float2 cs) {
  x = bf16_round(x);
  y = bf16_round(y);
  const float re = __fadd_rn(__fmul_rn(x, cs.x), __fmul_rn(y, cs.y));
  const float im = __fsub_rn(__fmul_rn(y, cs.x), __fmul_rn(x, cs.y));
  x = re;
  y = im;
}

// All lanes wait; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// NH consecutive TMEM columns of this thread's lane into v (32x32b shape).
template <int NH>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
  if constexpr (NH == 16) {
    tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
    tmem_ld_wait_regs16(v);
  } else {
#pragma unroll
    for (int c = 0; c < NH / 32; c++)
      tmem_ld32(taddr + c * 32, *reinterpret_cast<float(*)[32]>(v + 32 * c));
#pragma unroll
    for (int c = 0; c < NH / 32; c++) tmem_ld_wait_regs(v + 32 * c);
  }
}

template <int NH, int DQK, bool kFp8>
__global__ void __launch_bounds__(kThreads, 1)
    attn_gather_sm100_kernel(const __grid_constant__ GatherParams p) {
  using C = GCfg<NH, DQK>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* sQ = smem_raw + pad;
  uint8_t* sKV = sQ + C::kQBytes;
  uint8_t* sP = sKV + 2 * C::kSlotBytes;
  float* sS = reinterpret_cast<float*>(sP + C::kPBytes);
  GatherShared* sh = reinterpret_cast<GatherShared*>(sS + NH * kTok);
  volatile int* abort = &sh->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // the work unit: query row, head group, KV split
  const int64_t unit = blockIdx.x;
  const int split = (int)(unit % p.splits);
  const int64_t rest = unit / p.splits;
  const int hg = (int)(rest % p.hgroups);
  const int64_t row = rest / p.hgroups;
  const int64_t bidx = row / p.s, tpos = row % p.s;
  const bool paged = p.table != nullptr;
  // paged: query t of s sees the cached prefix up to its own position
  const int64_t len = paged ? (int64_t)p.seqlens[bidx] - (p.s - 1 - tpos) : p.topk;
  const int64_t ntiles = len > 0 ? (len + kTok - 1) / kTok : 0;
  const int t_begin = (int)(ntiles * split / p.splits);
  const int T = (int)(ntiles * (split + 1) / p.splits) - t_begin;
  const int h0 = hg * NH;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&sh->kv_full[i], kGroupWarps * 32);
      mbar_init(&sh->kv_empty[i], 1);
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_free[i], 4);
    }
    mbar_init(&sh->q_full, kGroupWarps * 32);
    mbar_init(&sh->p_full, 4);
    mbar_init(&sh->p_free, 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->xa, 4);
    mbar_init(&sh->xb, 4);
    mbar_init(&sh->xc, 4);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == kQkWarp) tmem_alloc<1>(&sh->tmem_base, C::kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp >= kProd0) {
    // ------------------------------------------------ producers
    const int grp = (warp - kProd0) / kGroupWarps;
    const int pw = (warp - kProd0) % kGroupWarps;
    const int gt = threadIdx.x - (kProd0 + grp * kGroupWarps) * 32;  // 0..127 in the group
    if (grp == 0) {
      // Q of the head group: NH rows of d_qk values, K-major chunks [NH][128 B]
      for (int i = gt; i < NH * (DQK / 8); i += kGroupWarps * 32) {
        const int r = i / (DQK / 8), u = i % (DQK / 8);
        const uint32_t dst = smem_u32(sQ + (u >> 3) * (NH * 128) + r * 128 + (((u & 7) ^ (r & 7)) << 4));
        if (h0 + r < p.h && T > 0)
          cp_async16(dst, p.q + (row * p.h + h0 + r) * p.q_row_stride + u * 8);
        else
          st_shared16(dst, make_uint4(0u, 0u, 0u, 0u));
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&sh->q_full);
    }
    bool ok = true;
    for (int n = grp; n < T && ok; n += 2) {
      const int64_t t0 = (int64_t)(t_begin + n) * kTok;
      // lane k < 16 resolves row pw + 4k of the tile: its latent row, or -1
      int64_t my_row = -1;
      float my_scale = 0.f;
      if (lane < 16) {
        const int64_t j = t0 + pw + 4 * lane;
        if (j < len) {
          if (paged) {
            const int64_t col = j / p.page_size;
            const int64_t pg = col < p.max_pages ? p.table[bidx * p.max_pages + col] : -1;
            if (pg >= 0 && pg < p.num_pages)
              my_row = pg * p.page_size + j % p.page_size;
            else
              raise_dev_error(p.err, QCAU_DEVERR_INDEX);
          } else {
            const int64_t id = p.idx[row * p.topk + j];
            if (id >= 0 && id < p.n_kv) my_row = bidx * p.n_kv + id;
          }
        }
        if (kFp8 && my_row >= 0) my_scale = __ldg(p.kv_scale + my_row);
      }
      // FP8: the codes are loaded before the slot is free (lane l: codes
      // [16l, 16l+16) of each of the warp's 16 rows)
      uint4 codes[kFp8 ? 16 : 1];
      if constexpr (kFp8) {
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const int64_t rr = shfl_i64(my_row, k);
          codes[k] = rr >= 0 ? ldg_nc16(p.kv_fp8 + rr * 512 + lane * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      // slot grp is free once PV of tile n - 2 has completed
      if (n >= 2 && !(ok = warp_wait(&sh->kv_empty[grp], ((n >> 1) - 1) & 1, abort))) break;
      uint8_t* slot = sKV + grp * C::kSlotBytes;
      if (lane < 16) sh->valid[grp][pw + 4 * lane] = my_row >= 0 ? 1 : 0;
      if constexpr (kFp8) {
        // dims [16l, 16l+16) = chunk l/4, 16-byte units 2(l%4) and 2(l%4)+1;
        // odd chunks store their second unit first (no bank conflicts)
        const int c = lane >> 2, u0 = 2 * (lane & 3);
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const int r = pw + 4 * k;
          const float sc = __shfl_sync(0xffffffffu, my_scale, k);
          const uint4 lo = e4m3x8_to_bf16(codes[k].x, codes[k].y, sc);
          const uint4 hi = e4m3x8_to_bf16(codes[k].z, codes[k].w, sc);
          const uint32_t rb = smem_u32(slot + c * 8192 + r * 128);
          const uint32_t a0 = rb + ((u0 ^ (r & 7)) << 4), a1 = rb + (((u0 + 1) ^ (r & 7)) << 4);
          if (c & 1) {
            st_shared16(a1, hi);
            st_shared16(a0, lo);
          } else {
            st_shared16(a0, lo);
            st_shared16(a1, hi);
          }
        }
        // rope part: chunk 8, 8 units a row; lane l takes unit l%8 of rows
        // pw + 4(l/8 + 4j)
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const int k = (lane >> 3) + 4 * jj, u = lane & 7, r = pw + 4 * k;
          const int64_t rr = shfl_i64(my_row, k);
          const uint32_t dst = smem_u32(slot + 8 * 8192 + r * 128 + ((u ^ (r & 7)) << 4));
          if (rr >= 0)
            cp_async16(dst, p.kv_rope + rr * 64 + u * 8);
          else
            st_shared16(dst, make_uint4(0u, 0u, 0u, 0u));
        }
      } else {
        // bf16 rows: DQK/8 units a row; lane l takes units l, l + 32 (, l + 64)
#pragma unroll 4
        for (int k = 0; k < 16; k++) {
          const int r = pw + 4 * k;
          const int64_t rr = shfl_i64(my_row, k);
          const __nv_bfloat16* src = p.kv + (rr >= 0 ? rr : 0) * p.d_kv;
#pragma unroll
          for (int u = lane; u < DQK / 8; u += 32) {
            const uint32_t dst =
                smem_u32(slot + (u >> 3) * 8192 + r * 128 + (((u & 7) ^ (r & 7)) << 4));
            if (rr >= 0)
              cp_async16(dst, src + u * 8);
            else
              st_shared16(dst, make_uint4(0u, 0u, 0u, 0u));
          }
        }
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&sh->kv_full[grp]);
    }
    cp_async_wait_all();
  } else if (warp == kQkWarp) {
    // ------------------------------------------------ QK issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(64, NH, kFmtBF16, kFmtBF16, false, false);
      const uint32_t q_addr = smem_u32(sQ), kv_addr = smem_u32(sKV);
      uint64_t* last = nullptr;
      int last_phase = 0;
      bool ok = true;
      for (int n = 0; n < T && ok; n++) {
        const int b = n & 1;
        if (n == 0 && !(ok = mbar_wait(&sh->q_full, 0, abort))) break;
        if (!(ok = mbar_wait(&sh->kv_full[b], (n >> 1) & 1, abort))) break;
        if (n >= 2 && !(ok = mbar_wait(&sh->s_free[b], ((n >> 1) - 1) & 1, abort))) break;
        tc_fence_after();
        const uint32_t slot = kv_addr + b * C::kSlotBytes;
#pragma unroll
        for (int c = 0; c < C::kChunks; c++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_bf16(tmem + C::kColS + b * NH, make_sdesc(slot + c * 8192 + kk * 32, 16, 1024),
                     make_sdesc(q_addr + c * (NH * 128) + kk * 32, 16, 1024), idesc,
                     (c | kk) != 0 ? 1u : 0u);
        tc_commit(&sh->s_full[b]);
        last = &sh->s_full[b];
        last_phase = (n >> 1) & 1;
      }
      if (*abort && last != nullptr) {
        volatile int never = 0;
        mbar_wait(last, last_phase, &never);
      }
    }
    __syncwarp();
  } else if (warp == kPvWarp) {
    // ------------------------------------------------ PV issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, NH, kFmtBF16, kFmtBF16, true, false);
      const uint32_t p_addr = smem_u32(sP), kv_addr = smem_u32(sKV);
      uint64_t* last = nullptr;
      int last_phase = 0;
      bool ok = true;
      for (int n = 0; n < T && ok; n++) {
        if (!(ok = mbar_wait(&sh->p_full, n & 1, abort))) break;
        tc_fence_after();
        const uint32_t slot = kv_addr + (n & 1) * C::kSlotBytes;
        // block j: dims [128j, 128j+128) = chunks 2j, 2j+1 (8192 bytes apart),
        // 16 rows (2048 bytes) per MMA
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_bf16(tmem + C::kColO + j * NH,
                     make_sdesc(slot + 2 * j * 8192 + kk * 2048, 8192, 1024),
                     make_sdesc(p_addr + kk * 32, 16, 1024), idesc,
                     (n > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sh->p_free);
        tc_commit(&sh->kv_empty[n & 1]);
        last = &sh->p_free;
        last_phase = n & 1;
      }
      if (ok && T > 0) tc_commit(&sh->o_full);
      if (*abort && last != nullptr) {
        volatile int never = 0;
        mbar_wait(last, last_phase, &never);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax / epilogue
    const int tid = threadIdx.x;             // TMEM lane of O^T (a latent dim of each block)
    const int hh = tid / C::kTph, g = tid % C::kTph;  // softmax stage: head, row group
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    float m_run = -INFINITY, l_part = 0.f;
    bool ok = true;
    for (int n = 0; n < T && ok; n++) {
      const int b = n & 1;
      if (!(ok = warp_wait(&sh->s_full[b], (n >> 1) & 1, abort))) break;
      if (!(ok = warp_wait(&sh->kv_full[b], (n >> 1) & 1, abort))) break;  // valid flags
      tc_fence_after();
      {
        float v[NH];
        tmem_ld_cols<NH>(tmem + lane_base + C::kColS + b * NH, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->s_free[b]);
        if (lane < 16) {
          const int m = 16 * warp + lane;  // the tile row in this TMEM lane (M = 64 layout)
#pragma unroll
          for (int h = 0; h < NH; h++) sS[h * kTok + m] = v[h];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->xa);
      if (!(ok = warp_wait(&sh->xa, n & 1, abort))) break;
      // head hh, rows [g * kTpt, +kTpt)
      float s[C::kTpt];
#pragma unroll
      for (int i = 0; i < C::kTpt; i += 4) {
        const float4 f = *reinterpret_cast<const float4*>(sS + hh * kTok + g * C::kTpt + i);
        s[i] = f.x;
        s[i + 1] = f.y;
        s[i + 2] = f.z;
        s[i + 3] = f.w;
      }
      const int* vld = sh->valid[b] + g * C::kTpt;
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < C::kTpt; i++)
        if (vld[i]) mx = fmaxf(mx, s[i]);
#pragma unroll
      for (int o = 1; o < C::kTph; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mx = mx == -INFINITY ? -INFINITY : mx * sl2;
      const float m_new = fmaxf(m_run, mx);
      float alpha = 1.f;
      if (m_new != m_run) alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
      m_run = m_new;
      uint32_t pk[C::kTpt / 2];
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < C::kTpt; i += 2) {
        float p0 = 0.f, p1 = 0.f;
        if (m_new != -INFINITY) {
          if (vld[i]) p0 = ex2_approx(fmaf(s[i], sl2, -m_new));
          if (vld[i + 1]) p1 = ex2_approx(fmaf(s[i + 1], sl2, -m_new));
        }
        psum += p0 + p1;
        __nv_bfloat162 t2 = __floats2bfloat162_rn(p0, p1);
        pk[i / 2] = *reinterpret_cast<uint32_t*>(&t2);
      }
      l_part = l_part * alpha + psum;
      if (g == 0) sh->alpha[hh] = alpha;
      const bool any = __any_sync(0xffffffffu, alpha != 1.f);
      if (lane == 0) {
        sh->resc[warp] = any ? 1 : 0;
        mbar_arrive(&sh->xb);
      }
      if (!(ok = warp_wait(&sh->xb, n & 1, abort))) break;
      const bool resc = (sh->resc[0] | sh->resc[1] | sh->resc[2] | sh->resc[3]) != 0;
      // P^T of tile n reuses the buffer of tile n-1, and O^T holds tiles < n,
      // once PV(n-1) is done
      if (n >= 1 && !(ok = warp_wait(&sh->p_free, (n - 1) & 1, abort))) break;
#pragma unroll
      for (int u = 0; u < C::kTpt / 8; u++) {
        const int unit = g * (C::kTpt / 8) + u;
        st_shared16(smem_u32(sP + hh * 128 + ((unit ^ (hh & 7)) << 4)),
                    make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]));
      }
      if (resc && n >= 1) {
        // O^T column c (block c / NH, head c % NH) of this lane times alpha
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < 4 * NH; c0 += 32) {
          float o[32];
          tmem_ld32(tmem + lane_base + C::kColO + c0, o);
          tmem_ld_wait_regs(o);
#pragma unroll
          for (int i = 0; i < 32; i++) o[i] *= sh->alpha[(c0 + i) % NH];
          tmem_st32(tmem + lane_base + C::kColO + c0, o);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->p_full);
    }
    if (ok && T > 0) ok = warp_wait(&sh->o_full, 0, abort);
    // per head: running max and denominator (the kTph threads' partial sums)
    float l_tot = l_part;
#pragma unroll
    for (int o = 1; o < C::kTph; o <<= 1) l_tot += __shfl_xor_sync(0xffffffffu, l_tot, o);
    const bool direct = p.splits == 1;
    if (g == 0) {
      sh->m_fin[hh] = m_run;
      if (direct) {
        // O / (l + 2^(sink log2e - m)), as attn_combine does for one part
        const int head = h0 + hh;
        const bool has_sink = p.sink != nullptr && head < p.h;
        const float sk = has_sink ? p.sink[head] * kLog2e : -INFINITY;
        float den;
        if (m_run != -INFINITY)
          den = l_tot + exp2f(sk - m_run);
        else
          den = l_tot + ((has_sink && isfinite(p.sink[head])) ? 1.f : 0.f);
        sh->l_fin[hh] = 1.f / fmaxf(den, 1.17549435e-38f);
      } else {
        sh->l_fin[hh] = l_tot;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->xc);
    if (ok) ok = warp_wait(&sh->xc, 0, abort);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < 4 * NH; c0 += 16) {
        float o[16];
        if (T > 0) {
          tmem_ld16(tmem + lane_base + C::kColO + c0, o);
          tmem_ld_wait_regs16(o);
        } else {
#pragma unroll
          for (int i = 0; i < 16; i++) o[i] = 0.f;
        }
        // 16 columns of one block (NH is a multiple of 16): dim 128 j + tid
        const int j = c0 / NH;
        const int dim = 128 * j + tid;
        if (direct) {
          const bool rope = p.inv_rope && dim >= 512 - p.rope_dim;
          float2 cs = make_float2(1.f, 0.f);
          if (rope)
            cs = reinterpret_cast<const float2*>(p.freqs)[(p.pos0 + tpos) * (p.rope_dim / 2) +
                                                          (dim - (512 - p.rope_dim)) / 2];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int h = (c0 + i) % NH;
            float x = o[i] * sh->l_fin[h];
            const float other = __shfl_xor_sync(0xffffffffu, x, 1);  // the pair's other dim
            if (rope) {
              float re = (lane & 1) ? other : x, im = (lane & 1) ? x : other;
              inv_rope(re, im, cs);
              x = (lane & 1) ? im : re;
            }
            if (h0 + h < p.h) p.out[(row * p.h + h0 + h) * 512 + dim] = __float2bfloat16_rn(x);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int h = (c0 + i) % NH;
            if (h0 + h < p.h)
              p.part_o[((row * p.splits + split) * p.h + h0 + h) * 512 + dim] = o[i];
          }
        }
      }
      if (!direct && g == 0 && h0 + hh < p.h) {
        const int64_t prow = (row * p.splits + split) * p.h + h0 + hh;
        p.part_ml[prow * 2] = m_run;
        p.part_ml[prow * 2 + 1] = sh->l_fin[hh];
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kQkWarp) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, C::kCols);
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(p.err, QCAU_DEVERR_TIMEOUT);
}

bool sm100_device() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

template <int NH, int DQK, bool kFp8>
cudaError_t launch_t(const GatherParams& p, int64_t units, cudaStream_t st) {
  using C = GCfg<NH, DQK>;
  cudaError_t e = cudaFuncSetAttribute(attn_gather_sm100_kernel<NH, DQK, kFp8>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  if (e != cudaSuccess) return e;
  attn_gather_sm100_kernel<NH, DQK, kFp8><<<(unsigned)units, kThreads, C::kSmem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

int gather_heads_per_cta(int64_t h, int64_t d_qk) {
  if (h <= 16) return 16;
  if (h <= 32 || d_qk == 576) return 32;
  return 64;
}

bool attn_gather_sm100_supported(const AttnArgs& a) {
  const bool fp8 = a.kv_fp8 != nullptr;
  const bool paged = a.block_table != nullptr;
  const bool widths = a.d_v == 512 && (a.d_qk == 512 || a.d_qk == 576) &&
                      (fp8 ? (a.d_qk == 576 && !paged && a.kv_scale && a.kv_rope)
                           : (a.d_kv >= a.d_qk && a.d_kv % 8 == 0 && a.kv != nullptr));
  const bool mode = paged ? (a.seqlens != nullptr && a.page_size > 0) : a.idx != nullptr;
  const bool plain = a.q_hblock <= 0 && a.part_hblock <= 0 && a.o_hblock <= 0 && !a.peer &&
                     a.splits_total <= 0 && !a.part_split_major && !a.part_f16;
  const bool rope = !a.inv_rope || (a.freqs != nullptr && a.rope_dim > 0 && a.rope_dim <= 512 &&
                                    a.rope_dim % 2 == 0);
  const bool aligned = (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && a.q_row_stride % 8 == 0 &&
                       (fp8 ? ((reinterpret_cast<uintptr_t>(a.kv_fp8) |
                                reinterpret_cast<uintptr_t>(a.kv_rope)) & 15) == 0
                            : (reinterpret_cast<uintptr_t>(a.kv) & 15) == 0);
  return widths && mode && plain && rope && aligned && a.h > 0 && a.splits >= 1 &&
         (a.splits == 1 || (a.part_o != nullptr && a.part_ml != nullptr)) && sm100_device();
}

cudaError_t launch_attn_gather_sm100(const AttnArgs& a, cudaStream_t st) {
  if (!attn_gather_sm100_supported(a)) return cudaErrorNotSupported;
  const int64_t rows = a.b * a.s;
  if (rows == 0) return cudaSuccess;
  GatherParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.q_row_stride = a.q_row_stride;
  p.kv = reinterpret_cast<const __nv_bfloat16*>(a.kv);
  p.kv_fp8 = a.kv_fp8;
  p.kv_scale = a.kv_scale;
  p.kv_rope = reinterpret_cast<const __nv_bfloat16*>(a.kv_rope);
  p.idx = a.idx;
  p.table = a.block_table;
  p.seqlens = a.seqlens;
  p.sink = a.sink;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.part_o = a.part_o;
  p.part_ml = a.part_ml;
  p.freqs = a.freqs;
  p.err = device_error_word();
  p.rows = rows;
  p.s = a.s;
  p.h = a.h;
  p.n_kv = a.n_kv;
  p.topk = a.topk;
  p.d_kv = a.d_kv;
  p.page_size = a.page_size;
  p.max_pages = a.max_pages;
  p.num_pages = a.num_pages;
  p.pos0 = a.pos0;
  p.splits = a.splits;
  p.inv_rope = a.splits == 1 ? a.inv_rope : 0;  // with partials the combine rotates
  p.rope_dim = a.rope_dim;
  p.scale = a.scale;
  const int nh = gather_heads_per_cta(a.h, a.d_qk);
  p.hgroups = (int)((a.h + nh - 1) / nh);
  const int64_t units = rows * p.hgroups * a.splits;
  const bool fp8 = a.kv_fp8 != nullptr;
  if (fp8) {
    if (nh == 16) return launch_t<16, 576, true>(p, units, st);
    return launch_t<32, 576, true>(p, units, st);
  }
  if (a.d_qk == 576) {
    if (nh == 16) return launch_t<16, 576, false>(p, units, st);
    return launch_t<32, 576, false>(p, units, st);
  }
  if (nh == 16) return launch_t<16, 512, false>(p, units, st);
  if (nh == 32) return launch_t<32, 512, false>(p, units, st);
  return launch_t<64, 512, false>(p, units, st);
}

}  // namespace qcau
