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
// One CTA = one query row x one group of NH heads (16 or 32) x one KV split.
// Every gathered row is loaded once per head group, and the heads are the N
// dimension of both MMAs, so a 16-head shard does not pad the tensor work.
// At that N a tcgen05 MMA costs its issue floor (about 52 cycles for N <= 32
// on B200, whatever M), so the tile is as tall as one MMA allows:
//   QK : kind::f16, M = 128 gathered rows, N = NH, K = d_qk in 64-value
//        chunks: S^T in TMEM, lane = row, a column per head, two buffers;
//   PV : M = 128 latent dims (4 MMAs cover 512), N = NH, K = 128 rows:
//        A = the staged rows read MN-major (dims contiguous), B = P^T
//        (K-major [head][row]); O^T in TMEM, lane = dim, a column per head.
// Staging: 64-value chunks of 128 rows, 128-byte swizzled ([128 rows][128 B],
// the UMMA K-major layout), in a ring of 10 value chunks (the 8 of a tile
// plus 2: a PV block frees a chunk pair, which the next tile's chunks 2..7
// fill in order, so its QK follows PV block by block) and a small ring for
// the rope chunk (dims 512..575).  Producers: 8 warps, two lanes a row; FP8
// rows go through registers (codes, rope and scale of the next tile are
// loaded while the current one computes, converted chunk by chunk as the
// ring frees), bf16 rows by 16-byte cp.async.  Softmax: a thread per row;
// per-head maxima by a halving butterfly (lane l ends with head l), then
// NH threads update the running max; a tile that raises a head's max
// rescales that head's O^T column.
// Warps: 0-3 softmax / epilogue, 4 QK issuer + TMEM allocator, 5 PV issuer,
// 6-13 producers.
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

constexpr int kTok = 128;       // gathered rows per tile
constexpr int kVSlots = 10;     // value-chunk ring
constexpr int kChunkBytes = kTok * 128;
constexpr int kQkWarp = 4;
constexpr int kPvWarp = 5;
constexpr int kProd0 = 6;       // first producer warp
constexpr int kProdWarps = 8;
constexpr int kThreads = (kProd0 + kProdWarps) * 32;  // 448
constexpr float kLog2e = 1.4426950408889634f;

struct GatherShared {
  uint64_t vfull[kVSlots];   // value chunk staged (256 producer threads)
  uint64_t vempty[kVSlots];  // PV done with it
  uint64_t rfull[2];         // rope chunk staged
  uint64_t rempty[2];        // QK done with it
  uint64_t q_full;           // Q staged
  uint64_t s_full[2];        // QK done into S^T buffer b
  uint64_t s_free[2];        // the 4 softmax warps read S^T buffer b
  uint64_t p_full;           // P^T written and O^T rescaled (4 softmax warps)
  uint64_t p_free;           // PV done with P^T and O^T
  uint64_t o_full;           // last PV done
  uint64_t xa, xb, xc, xd;   // softmax warps: maxima / running max / sums / finals
  int valid[2][kTok];
  float xmax[4][32];
  float xsum[4][32];
  float m_cur[32];
  float alpha[32];
  float fin[32];
  int resc;
  uint32_t tmem_base;
  int abort;
};

template <int NH, int DQK>
struct GCfg {
  static constexpr int kRSlots = DQK == 576 ? (NH == 16 ? 2 : 1) : 0;
  static constexpr int kQBytes = NH * DQK * 2;         // [chunk][NH rows][128 B]
  static constexpr int kPBytes = 2 * NH * 128;         // P^T [2 row halves][NH rows][128 B]
  static constexpr uint32_t kColO = 0;                 // O^T: 4 blocks of NH columns
  static constexpr uint32_t kColS = 4 * NH;            // S^T: 2 buffers of NH columns
  static constexpr uint32_t kCols = 6 * NH <= 128 ? 128 : 256;
  static constexpr size_t kSmem = 1024 + (size_t)kQBytes + (size_t)(kVSlots + kRSlots) * kChunkBytes +
                                  kPBytes + sizeof(GatherShared);
  static_assert(NH == 16 || NH == 32, "heads per CTA");
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
__device__ __forceinline__ void st_shared_u16(uint32_t dst, uint16_t v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(dst), "h"(v) : "memory");
}
// 32 bytes (32-byte aligned) by one 256-bit load
__device__ __forceinline__ void ldg_nc32(const void* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z),
                 "=r"(hi.w)
               : "l"(p));
}
__device__ __forceinline__ uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
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

// All lanes wait; the warp agrees on the outcome.  (Lane 0 alone waiting,
// then __syncwarp, measured slower here and in the decode kernel.)
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
    tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(v));
    tmem_ld_wait_regs(v);
  }
}

// Per-head reduction of v[NH] over the warp's 32 lanes by halving exchanges:
// at each step a lane keeps half of its heads and takes the partner's
// values of them.  Returns the result for head lane (NH = 32) or lane / 2
// (NH = 16).  kMax: max, else sum.
template <int NH, bool kMax>
__device__ __forceinline__ float warp_head_reduce(float* v, int lane) {
  int n = NH;
#pragma unroll
  for (int m = 16; m >= 1 && n > 1; m >>= 1) {
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      if (i < n / 2) {
        const float send = up ? v[i] : v[i + n / 2];
        const float keep = up ? v[i + n / 2] : v[i];
        const float got = __shfl_xor_sync(0xffffffffu, send, m);
        v[i] = kMax ? fmaxf(keep, got) : keep + got;
      }
    }
    n >>= 1;
  }
  float r = v[0];
  if constexpr (NH == 16) {  // lanes l and l ^ 1 hold head l / 2 over other rows
    const float got = __shfl_xor_sync(0xffffffffu, r, 1);
    r = kMax ? fmaxf(r, got) : r + got;
  }
  return r;
}

// 14 warps: the sub-partition that runs four of them holds 4 x 32 x 128
// registers, its whole register file.
template <int NH, int DQK, bool kFp8>
__global__ void __launch_bounds__(kThreads, 1)
    attn_gather_sm100_kernel(const __grid_constant__ GatherParams p) {
  using C = GCfg<NH, DQK>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* sQ = smem_raw + pad;
  uint8_t* sV = sQ + C::kQBytes;
  uint8_t* sR = sV + kVSlots * kChunkBytes;
  uint8_t* sP = sR + C::kRSlots * kChunkBytes;
  GatherShared* sh = reinterpret_cast<GatherShared*>(sP + C::kPBytes);
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
    for (int i = 0; i < kVSlots; i++) {
      mbar_init(&sh->vfull[i], kProdWarps * 32);
      mbar_init(&sh->vempty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&sh->rfull[i], kProdWarps * 32);
      mbar_init(&sh->rempty[i], 1);
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_free[i], 4);
    }
    mbar_init(&sh->q_full, kProdWarps * 32);
    mbar_init(&sh->p_full, 4);
    mbar_init(&sh->p_free, 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->xa, 4);
    mbar_init(&sh->xb, 4);
    mbar_init(&sh->xc, 4);
    mbar_init(&sh->xd, 4);
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
    const int pt = threadIdx.x - kProd0 * 32;        // 0..255
    const int prow = 16 * (warp - kProd0) + (lane >> 1), half = lane & 1;
    const uint32_t row_sw = (uint32_t)(prow & 7);
    // Q of the head group: NH rows of d_qk values, K-major chunks [NH][128 B]
    for (int i = pt; i < NH * (DQK / 8); i += kProdWarps * 32) {
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

    // key of this thread's row in tile n: the top-k index, or the block-table
    // entry of its page; `has` = the row exists in the key list
    auto load_key = [&](int n, bool& has) -> int64_t {
      const int64_t j = (int64_t)(t_begin + n) * kTok + prow;
      has = j < len;
      if (!has) return -1;
      if (paged) {
        const int64_t col = j / p.page_size;
        return col < p.max_pages ? (int64_t)p.table[bidx * p.max_pages + col] : -1;
      }
      return (int64_t)p.idx[row * p.topk + j];
    };
    // latent row of the key, or -1 (a masked key)
    auto row_of = [&](int n, int64_t key, bool has) -> int64_t {
      if (!has) return -1;
      if (paged) {
        if (key >= 0 && key < p.num_pages) {
          const int64_t j = (int64_t)(t_begin + n) * kTok + prow;
          return key * p.page_size + j % p.page_size;
        }
        if (half == 0) raise_dev_error(p.err, QCAU_DEVERR_INDEX);
        return -1;
      }
      return (key >= 0 && key < p.n_kv) ? bidx * p.n_kv + key : -1;
    };

    // bf16 rows: a tile's rows are prefetched into L2 one tile ahead of their
    // copies (keys two tiles ahead).  FP8 rows: the codes of chunk c of the
    // next tile are loaded into the registers of chunk c as soon as this
    // tile's chunk c is stored, a tile ahead of their use, so the loads are
    // spread over the tile instead of queued together (a burst of them stalls
    // the softmax warps' shared-memory accesses behind it)
    auto prefetch_row = [&](int64_t r) {
      if (r >= 0) prefetch_l2(p.kv + r * p.d_kv + half * (DQK / 2), DQK);  // half a row
    };
    bool ok = true;
    bool has = false, has1 = false;
    int64_t key = T > 0 ? load_key(0, has) : -1;
    int64_t key1 = T > 1 ? load_key(1, has1) : -1;
    // FP8: codes [64c + 32 half, +32) of chunk c of the tile in codes[2c],
    // codes[2c+1] (one 32-byte load: the row's two lanes read 64 contiguous
    // bytes), and the row's scale
    uint4 codes[kFp8 ? 16 : 1];
    float sc = 0.f;
    auto load_codes = [&](int64_t r, float& scale_out) {
      if constexpr (kFp8) {
        if (r >= 0) {
          const uint8_t* src = p.kv_fp8 + r * 512 + 32 * half;
#pragma unroll
          for (int c = 0; c < 8; c++) ldg_nc32(src + 64 * c, codes[2 * c], codes[2 * c + 1]);
          scale_out = __ldg(p.kv_scale + r);
        } else {
#pragma unroll
          for (int c = 0; c < 16; c++) codes[c] = make_uint4(0u, 0u, 0u, 0u);
          scale_out = 0.f;
        }
      }
    };
    if constexpr (kFp8) {
      load_codes(row_of(0, key, has), sc);
    } else {
      prefetch_row(row_of(0, key, has));
    }
    for (int n = 0; n < T && ok; n++) {
      const int64_t rr = row_of(n, key, has);
      const int64_t rn = n + 1 < T ? row_of(n + 1, key1, has1) : -1;  // next tile's row
      if constexpr (!kFp8) {
        if (n + 1 < T) prefetch_row(rn);
      }
      float sc_next = 0.f;
      if constexpr (kFp8) {
        if (rn >= 0) sc_next = __ldg(p.kv_scale + rn);
      }
      bool has2 = false;
      const int64_t key2 = n + 2 < T ? load_key(n + 2, has2) : -1;
      // rope chunk (dims 512..575): bf16 in both formats, copied as soon as
      // its ring slot is free (QK of the tile before has read it)
      const int rs = DQK == 576 ? n % C::kRSlots : 0, ru = DQK == 576 ? n / C::kRSlots : 0;
      if constexpr (DQK == 576) {
        if (ru >= 1 && !(ok = warp_wait(&sh->rempty[rs], (ru - 1) & 1, abort))) break;
        const __nv_bfloat16* src = kFp8 ? p.kv_rope + (rr >= 0 ? rr : 0) * 64
                                        : p.kv + (rr >= 0 ? rr : 0) * p.d_kv + 512;
        uint8_t* dstrow = sR + rs * kChunkBytes + prow * 128;
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t dst = smem_u32(dstrow + (((uint32_t)(4 * half + i) ^ row_sw) << 4));
          if (rr >= 0)
            cp_async16(dst, src + 32 * half + 8 * i);
          else
            st_shared16(dst, make_uint4(0u, 0u, 0u, 0u));
        }
      }
      const __nv_bfloat16* brow = kFp8 ? nullptr : p.kv + (rr >= 0 ? rr : 0) * p.d_kv;
      // value chunks 0..7, each into the ring slot that PV has freed
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const int q = 8 * n + c, slot = q % kVSlots, u = q / kVSlots;
        if (u >= 1 && !(ok = warp_wait(&sh->vempty[slot], (u - 1) & 1, abort))) break;
        if (c == 0 && half == 0) sh->valid[n & 1][prow] = rr >= 0 ? 1 : 0;
        uint8_t* dstrow = sV + slot * kChunkBytes + prow * 128;
        if constexpr (kFp8) {
          if (c == 0 && DQK == 576) {
            // the rope copies of this tile have landed long since
            cp_async_wait_all();
            fence_proxy_async_smem();
            mbar_arrive(&sh->rfull[rs]);
          }
          // dims 64c + 32 half + [0, 32) -> units 4 half .. 4 half + 3
          const uint4 w0 = e4m3x8_to_bf16(codes[2 * c].x, codes[2 * c].y, sc);
          const uint4 w1 = e4m3x8_to_bf16(codes[2 * c].z, codes[2 * c].w, sc);
          const uint4 w2 = e4m3x8_to_bf16(codes[2 * c + 1].x, codes[2 * c + 1].y, sc);
          const uint4 w3 = e4m3x8_to_bf16(codes[2 * c + 1].z, codes[2 * c + 1].w, sc);
          const uint32_t u0 = (uint32_t)(4 * half);
          st_shared16(smem_u32(dstrow + ((u0 ^ row_sw) << 4)), w0);
          st_shared16(smem_u32(dstrow + (((u0 + 1) ^ row_sw) << 4)), w1);
          st_shared16(smem_u32(dstrow + (((u0 + 2) ^ row_sw) << 4)), w2);
          st_shared16(smem_u32(dstrow + (((u0 + 3) ^ row_sw) << 4)), w3);
          fence_proxy_async_smem();
          mbar_arrive(&sh->vfull[slot]);
          // refill: chunk c of the next tile
          if (rn >= 0) {
            ldg_nc32(p.kv_fp8 + rn * 512 + 32 * half + 64 * c, codes[2 * c], codes[2 * c + 1]);
          } else {
            codes[2 * c] = make_uint4(0u, 0u, 0u, 0u);
            codes[2 * c + 1] = make_uint4(0u, 0u, 0u, 0u);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const uint32_t dst = smem_u32(dstrow + (((uint32_t)(4 * half + i) ^ row_sw) << 4));
            if (rr >= 0)
              cp_async16(dst, brow + 64 * c + 32 * half + 8 * i);
            else
              st_shared16(dst, make_uint4(0u, 0u, 0u, 0u));
          }
        }
      }
      if (!ok) break;
      if constexpr (!kFp8) {
        // bf16 rows: the tile's copies land together
        cp_async_wait_all();
        fence_proxy_async_smem();
        if constexpr (DQK == 576) mbar_arrive(&sh->rfull[n % C::kRSlots]);
#pragma unroll 1
        for (int c = 0; c < 8; c++) mbar_arrive(&sh->vfull[(8 * n + c) % kVSlots]);
      }
      sc = sc_next;
      key = key1;
      has = has1;
      key1 = key2;
      has1 = has2;
    }
    cp_async_wait_all();
  } else if (warp == kQkWarp) {
    // ------------------------------------------------ QK issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, NH, kFmtBF16, kFmtBF16, false, false);
      const uint32_t q_addr = smem_u32(sQ), v_addr = smem_u32(sV), r_addr = smem_u32(sR);
      uint64_t* last = nullptr;
      int last_phase = 0;
      bool ok = true;
      for (int n = 0; n < T && ok; n++) {
        const int b = n & 1;
        if (n == 0 && !(ok = mbar_wait(&sh->q_full, 0, abort))) break;
        if (n >= 2 && !(ok = mbar_wait(&sh->s_free[b], ((n >> 1) - 1) & 1, abort))) break;
        bool first = true;
        if constexpr (DQK == 576) {
          // the rope chunk first: its ring is free ahead of the value chunks
          const int rs = n % C::kRSlots, ru = n / C::kRSlots;
          if (!(ok = mbar_wait(&sh->rfull[rs], ru & 1, abort))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_bf16(tmem + C::kColS + b * NH,
                     make_sdesc(r_addr + rs * kChunkBytes + kk * 32, 16, 1024),
                     make_sdesc(q_addr + 8 * (NH * 128) + kk * 32, 16, 1024), idesc,
                     kk != 0 ? 1u : 0u);
          tc_commit(&sh->rempty[rs]);
          first = false;
        }
#pragma unroll 1
        for (int c = 0; c < 8 && ok; c++) {
          const int q = 8 * n + c, slot = q % kVSlots, u = q / kVSlots;
          if (!(ok = mbar_wait(&sh->vfull[slot], u & 1, abort))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_bf16(tmem + C::kColS + b * NH,
                     make_sdesc(v_addr + slot * kChunkBytes + kk * 32, 16, 1024),
                     make_sdesc(q_addr + c * (NH * 128) + kk * 32, 16, 1024), idesc,
                     (first && kk == 0) ? 0u : 1u);
          first = false;
        }
        if (!ok) break;
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
      const uint32_t p_addr = smem_u32(sP), v_addr = smem_u32(sV);
      uint64_t* last = nullptr;
      int last_phase = 0;
      bool ok = true;
      for (int n = 0; n < T && ok; n++) {
        if (!(ok = mbar_wait(&sh->p_full, n & 1, abort))) break;
        tc_fence_after();
        // block j: dims [128j, +128) = value chunks 2j, 2j+1 of the tile, in
        // ring slots s0 and s0 + 1 (s0 even: a pair never wraps); 16 rows
        // (2048 bytes) a MMA
#pragma unroll 1
        for (int j = 0; j < 4; j++) {
          const int s0 = (8 * n + 2 * j) % kVSlots;
#pragma unroll
          for (int kk = 0; kk < 8; kk++)
            mma_bf16(tmem + C::kColO + j * NH,
                     make_sdesc(v_addr + s0 * kChunkBytes + kk * 2048, kChunkBytes, 1024),
                     make_sdesc(p_addr + (kk >> 2) * (NH * 128) + (kk & 3) * 32, 16, 1024),
                     idesc, (n > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh->vempty[s0]);
          tc_commit(&sh->vempty[s0 + 1]);
        }
        tc_commit(&sh->p_free);
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
    const int t = threadIdx.x;  // TMEM lane: tile row t of S^T, latent dim t of each O^T block
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    float m_run = -INFINITY;    // threads t < NH: running max of head t (log2 units)
    float l_part[NH];           // this row's share of each head's denominator
#pragma unroll
    for (int h = 0; h < NH; h++) l_part[h] = 0.f;
    bool ok = true;
    for (int n = 0; n < T && ok; n++) {
      const int b = n & 1;
      if (!(ok = warp_wait(&sh->s_full[b], (n >> 1) & 1, abort))) break;
      {  // the valid flags of the tile arrived with its first value chunk
        const int q0 = 8 * n;
        if (!(ok = warp_wait(&sh->vfull[q0 % kVSlots], (q0 / kVSlots) & 1, abort))) break;
      }
      tc_fence_after();
      float s[NH];
      tmem_ld_cols<NH>(tmem + lane_base + C::kColS + b * NH, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->s_free[b]);
      const bool vld = sh->valid[b][t] != 0;
      {
        float v[NH];
#pragma unroll
        for (int h = 0; h < NH; h++) v[h] = vld ? s[h] : -INFINITY;
        const float wm = warp_head_reduce<NH, true>(v, lane);
        if (NH == 32 || (lane & 1) == 0) sh->xmax[warp][NH == 32 ? lane : lane >> 1] = wm;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->xa);
      if (!(ok = warp_wait(&sh->xa, n & 1, abort))) break;
      if (warp == 0) {
        float alpha = 1.f;
        if (t < NH) {
          float tm = fmaxf(fmaxf(sh->xmax[0][t], sh->xmax[1][t]), fmaxf(sh->xmax[2][t], sh->xmax[3][t]));
          tm = tm == -INFINITY ? -INFINITY : tm * sl2;
          const float m_new = fmaxf(m_run, tm);
          if (m_new != m_run) alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
          m_run = m_new;
          sh->m_cur[t] = m_new;
          sh->alpha[t] = alpha;
        }
        const bool any = __any_sync(0xffffffffu, alpha != 1.f);
        if (lane == 0) sh->resc = any ? 1 : 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->xb);
      if (!(ok = warp_wait(&sh->xb, n & 1, abort))) break;
      const bool resc = sh->resc != 0;
      // P^T of tile n reuses the buffer of tile n-1, and O^T holds tiles < n,
      // once PV(n-1) is done
      if (n >= 1 && !(ok = warp_wait(&sh->p_free, (n - 1) & 1, abort))) break;
      {
        // P of this row for every head, stored as column t of P^T
        const uint32_t pbase = smem_u32(sP + (t >> 6) * (NH * 128)) + (t & 7) * 2;
        const uint32_t unit = (uint32_t)((t & 63) >> 3);
#pragma unroll
        for (int h = 0; h < NH; h++) {
          const float m = sh->m_cur[h];
          const float pv = (vld && m != -INFINITY) ? ex2_approx(fmaf(s[h], sl2, -m)) : 0.f;
          l_part[h] = l_part[h] * sh->alpha[h] + pv;
          st_shared_u16(pbase + h * 128 + ((unit ^ (uint32_t)(h & 7)) << 4),
                        __bfloat16_as_ushort(__float2bfloat16_rn(pv)));
        }
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
    // per head: the denominator over the 128 rows
    {
      const float ws = warp_head_reduce<NH, false>(l_part, lane);
      if (NH == 32 || (lane & 1) == 0) sh->xsum[warp][NH == 32 ? lane : lane >> 1] = ws;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->xc);
    if (ok) ok = warp_wait(&sh->xc, 0, abort);
    const bool direct = p.splits == 1;
    if (ok && t < NH) {
      const float l_tot = sh->xsum[0][t] + sh->xsum[1][t] + sh->xsum[2][t] + sh->xsum[3][t];
      if (direct) {
        // O / (l + 2^(sink log2e - m)), as attn_combine does for one part
        const int head = h0 + t;
        const bool has_sink = p.sink != nullptr && head < p.h;
        const float sk = has_sink ? p.sink[head] * kLog2e : -INFINITY;
        float den;
        if (m_run != -INFINITY)
          den = l_tot + exp2f(sk - m_run);
        else
          den = l_tot + ((has_sink && isfinite(p.sink[head])) ? 1.f : 0.f);
        sh->fin[t] = 1.f / fmaxf(den, 1.17549435e-38f);
      } else if (h0 + t < p.h) {
        const int64_t prow = (row * p.splits + split) * p.h + h0 + t;
        p.part_ml[prow * 2] = m_run;
        p.part_ml[prow * 2 + 1] = l_tot;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->xd);
    if (ok) ok = warp_wait(&sh->xd, 0, abort);
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
        // 16 columns of one block (NH is a multiple of 16): dim 128 j + t
        const int j = c0 / NH;
        const int dim = 128 * j + t;
        if (direct) {
          const bool rope = p.inv_rope && dim >= 512 - p.rope_dim;
          float2 cs = make_float2(1.f, 0.f);
          if (rope)
            cs = reinterpret_cast<const float2*>(p.freqs)[(p.pos0 + tpos) * (p.rope_dim / 2) +
                                                          (dim - (512 - p.rope_dim)) / 2];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const int h = (c0 + i) % NH;
            float x = o[i] * sh->fin[h];
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

int gather_heads_per_cta(int64_t h, int64_t /*d_qk*/) { return h <= 16 ? 16 : 32; }

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
                       (fp8 ? (reinterpret_cast<uintptr_t>(a.kv_fp8) & 31) == 0 &&
                                  (reinterpret_cast<uintptr_t>(a.kv_rope) & 15) == 0
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
  return launch_t<32, 512, false>(p, units, st);
}

}  // namespace qcau
