// bmm.cu -- batched bf16 GEMM on tcgen05 for the absorbed-MLA projections.
//
// The absorbed decode layer needs, per head h (batch index g = h):
//   absorb: q_lat[b, h, :]  = q_nope[b, h, :128] . W_UK[h]   (W_UK[h] = wkv_b
//           rows h*256 .. h*256+127, i.e. B given MN-major: N contiguous)
//   v-up  : o_v[b, h, :]    = o_lat[b, h, :512] . W_UV[h]^T (W_UV[h] rows
//           h*256+128 .. h*256+255, B given K-major: K contiguous)
// Both read their operands in place (strided 3-D TMA boxes) from the
// q-projection output, the attention output and wkv_b, so no transposes or
// copies are made.
//
// CTA = one 128 x BN output tile of one batch entry, 192 threads:
//   warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer,
//   warps 2-5 epilogue (TMEM -> bf16 rows).
// BN is 128, or 256 for the absorb (B MN-major, K = 128, N = 512): there
// 512 CTAs of 128 columns (128 heads x 4) took two waves of three CTAs per
// SM, each CTA a load, a short MMA chain and an epilogue in series; 256
// columns read the shared A tile once for twice the weight bytes and fit
// one wave of two CTAs per SM.
// Epilogue options: the act_quant of C in 1 x 128 blocks (the v-up, whose
// output rows are one head's 128 values), and the RoPE of a 64-value slice
// of another tensor per (row, batch entry) done under the MMAs (the absorb,
// for the query's rope part).
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int BM = 128, BK = 64;           // BK bf16 = 128-byte rows
constexpr int kTileBytes = 128 * BK * 2;   // 16 KB: A, or B at BN = 128
constexpr int kBChunk = 64 * BK * 2;       // 8 KB: 64 MN-major columns of B
constexpr int kThreads = 192;
template <int BN>
constexpr int stage_bytes() { return kTileBytes + BN * BK * 2; }

// Stages of the TMA ring: 2 when K fits in two steps (66 KB and three CTAs
// per SM at BN = 128; 98 KB and two CTAs per SM at BN = 256, the absorb);
// 4 for longer K (the v-up, K = 512).
template <int kStages>
struct BmmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull;
  uint32_t tmem_base;
  int abort;
};
template <int kStages, int BN>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)kStages * stage_bytes<BN>() + sizeof(BmmShared<kStages>);
}

// The epilogue's optional act_quant of C (one 128-wide block per tile row).
struct QuantOut {
  uint8_t* codes;
  void* scales;
  int round_scale, e8m0;
};

// The epilogue's optional RoPE of a 64-value slice per row (BmmArgs::rope_*).
struct RopeSide {
  __nv_bfloat16* x;
  __nv_bfloat16* copy;
  int64_t x_stride, copy_stride;
  const float* freqs;
  const int32_t* pos;
};

// One row's 32 (re, im) pairs, 16-byte loads and stores: the arithmetic of
// rope_pairs_kernel (rope_norm.cu) pair by pair.
__device__ __forceinline__ void rope_row64(__nv_bfloat16* x, __nv_bfloat16* copy,
                                           const float* fr) {
  uint4 v[8];
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = reinterpret_cast<const uint4*>(x)[i];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float4 f0 = reinterpret_cast<const float4*>(fr)[2 * i];
    const float4 f1 = reinterpret_cast<const float4*>(fr)[2 * i + 1];
    const float2 cs[4] = {make_float2(f0.x, f0.y), make_float2(f0.z, f0.w),
                          make_float2(f1.x, f1.y), make_float2(f1.z, f1.w)};
    uint32_t* w = reinterpret_cast<uint32_t*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[j]));
      const __nv_bfloat162 o =
          __floats2bfloat162_rn(__fsub_rn(__fmul_rn(a.x, cs[j].x), __fmul_rn(a.y, cs[j].y)),
                                __fadd_rn(__fmul_rn(a.x, cs[j].y), __fmul_rn(a.y, cs[j].x)));
      w[j] = *reinterpret_cast<const uint32_t*>(&o);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    reinterpret_cast<uint4*>(x)[i] = v[i];
    reinterpret_cast<uint4*>(copy)[i] = v[i];
  }
}

template <int kStages, int BN, bool kQuant, bool kRope>
__global__ void __launch_bounds__(kThreads, 1)
    bmm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
               int b_kmajor, __nv_bfloat16* __restrict__ c, int64_t c_bstride, int64_t c_rstride,
               int64_t m, int64_t k, QuantOut qo, RopeSide rp, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  constexpr int kStageBytes = stage_bytes<BN>();
  BmmShared<kStages>* sh =
      reinterpret_cast<BmmShared<kStages>*>(tiles + (size_t)kStages * kStageBytes);
  volatile int* abort = &sh->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, g = blockIdx.z;
  const int KS = (int)(k / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    mbar_init(&sh->tfull, 1);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<1>(&sh->tmem_base, BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0 && lane == 0) {
    int last_use[kStages];
    for (int s = 0; s < kStages; s++) last_use[s] = -1;
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % kStages, u = ks / kStages;
      if (!mbar_wait(&sh->empty[s], (u & 1) ^ 1, abort)) break;
      mbar_arrive_expect_tx(&sh->full[s], kStageBytes);
      uint8_t* st = tiles + (size_t)s * kStageBytes;
      tma_load_3d(st, &tm_a, &sh->full[s], ks * BK, m0, g);
      if (b_kmajor) {
        tma_load_3d(st + kTileBytes, &tm_b, &sh->full[s], ks * BK, n0, g);
      } else {
        // BN / 64 chunks of [64 K rows x 64 N = 128 B]
#pragma unroll
        for (int c = 0; c < BN / 64; c++)
          tma_load_3d(st + kTileBytes + c * kBChunk, &tm_b, &sh->full[s], n0 + 64 * c, ks * BK, g);
      }
      last_use[s] = u;
    }
    if (*abort) {
      volatile int never = 0;
      for (int s = 0; s < kStages; s++)
        if (last_use[s] >= 0) mbar_wait(&sh->full[s], last_use[s] & 1, &never);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = make_idesc(BM, BN, kFmtBF16, kFmtBF16, false, !b_kmajor);
    bool issued = false;
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % kStages, u = ks / kStages;
      if (!mbar_wait(&sh->full[s], u & 1, abort)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(tiles + (size_t)s * kStageBytes);
      const uint32_t b_addr = a_addr + kTileBytes;
#pragma unroll
      for (int kk = 0; kk < BK / 16; kk++) {
        const uint64_t ad = make_sdesc(a_addr + kk * 32, 16, 1024);
        const uint64_t bd = b_kmajor ? make_sdesc(b_addr + kk * 32, 16, 1024)
                                     : make_sdesc(b_addr + kk * 16 * 128, kBChunk, 1024);
        mma_bf16(tmem, ad, bd, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(&sh->empty[s]);
      issued = true;
    }
    if (issued) tc_commit(&sh->tfull);
    if (*abort && issued) {
      volatile int never = 0;
      mbar_wait(&sh->tfull, 0, &never);
    }
  } else if (warp >= 2) {
    const int quarter = warp & 3;
    const int64_t row = m0 + quarter * 32 + lane;
    if constexpr (kRope) {
      // the rope slice of this row and batch entry, once (the first N tile),
      // under the MMAs; the A tiles never cover it
      if (blockIdx.x == 0 && row < m) {
        const int64_t r = row * gridDim.z + g;
        rope_row64(rp.x + r * rp.x_stride, rp.copy + r * rp.copy_stride,
                   rp.freqs + (int64_t)rp.pos[row] * 64);
      }
    }
    // the TMEM loads below are warp-collective: the lanes decide together
    const bool landed = mbar_wait(&sh->tfull, 0, abort);
    if (__all_sync(0xffffffffu, landed)) {
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
      __nv_bfloat16* dst = c + g * c_bstride + row * c_rstride + n0;
      float amax = 0.f;  // of the row's bf16 outputs, for the act_quant
#pragma unroll
      for (int c4 = 0; c4 < BN / 32; c4++) {
        float v[32];
        __syncwarp();  // after the previous chunk's stores, which rows past m skip
        tmem_ld32(taddr + c4 * 32, v);
        tmem_ld_wait_regs(v);
        if constexpr (kQuant) {
#pragma unroll
          for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(bf16_round(v[j])));
        }
        if (row < m) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            uint4 pk;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * j + 0], v[8 * j + 1]);
            __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * j + 2], v[8 * j + 3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 4], v[8 * j + 5]);
            __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * j + 6], v[8 * j + 7]);
            pk.x = *reinterpret_cast<uint32_t*>(&h0);
            pk.y = *reinterpret_cast<uint32_t*>(&h1);
            pk.z = *reinterpret_cast<uint32_t*>(&h2);
            pk.w = *reinterpret_cast<uint32_t*>(&h3);
            d4[j] = pk;
          }
        }
      }
      if constexpr (kQuant) {
        // act_quant of the row's 128 bf16 values (act_quant.cu): the scale
        // from their absmax, then each value / scale, clamped, to e4m3.
        // tcgen05.ld is warp-collective: every lane loads, rows past m only
        // skip the stores.
        const float sc = act_scale(amax, qo.round_scale);
        uint8_t* cd = qo.codes + g * c_bstride + row * c_rstride + n0;
#pragma unroll
        for (int c4 = 0; c4 < BN / 32; c4++) {
          float v[32];
          __syncwarp();
          tmem_ld32(taddr + c4 * 32, v);
          tmem_ld_wait_regs(v);
          if (row < m) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
              uint32_t word = 0;
#pragma unroll
              for (int i = 0; i < 4; i++) {
                float q = __fdiv_rn(bf16_round(v[4 * j + i]), sc);
                q = fminf(fmaxf(q, -448.f), 448.f);
                word |= (uint32_t)f32_to_e4m3(q) << (8 * i);
              }
              w[j] = word;
            }
            uint4* d4 = reinterpret_cast<uint4*>(cd + c4 * 32);
            d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
        const int64_t si = row * (c_rstride / 128) + (g * c_bstride + n0) / 128;
        if (row < m) {
          if (qo.e8m0)
            reinterpret_cast<uint8_t*>(qo.scales)[si] = (uint8_t)((__float_as_uint(sc) >> 23) & 0xff);
          else
            reinterpret_cast<float*>(qo.scales)[si] = sc;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, BN);
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(err, QCAU_DEVERR_TIMEOUT);
}

}  // namespace

cudaError_t launch_bf16_bmm(const BmmArgs& p, cudaStream_t st) {
  if (p.m == 0 || p.batch == 0) return cudaSuccess;
  if (p.n % 128 || p.k % BK) return cudaErrorInvalidValue;
  const QuantOut qo{reinterpret_cast<uint8_t*>(p.q_codes), p.q_scales, p.q_round_scale,
                    p.q_scale_e8m0};
  if (qo.codes && (p.n != 128 || p.c_bstride % 128 || p.c_rstride % 128 || !p.q_scales))
    return cudaErrorInvalidValue;
  // 256-column tiles for an MN-major B with K of at most two steps (the
  // absorb); 128 otherwise (K-major B boxes stay 128 rows high)
  const RopeSide rp{reinterpret_cast<__nv_bfloat16*>(p.rope_x),
                    reinterpret_cast<__nv_bfloat16*>(p.rope_copy), p.rope_x_stride,
                    p.rope_copy_stride, p.rope_freqs, p.rope_pos};
  if (rp.x && (!rp.copy || !rp.freqs || !rp.pos || p.rope_x_stride % 8 ||
               p.rope_copy_stride % 8 || qo.codes))
    return cudaErrorInvalidValue;
  const bool wide = !p.b_kmajor && p.n % 256 == 0 && p.k / BK <= 2 && !qo.codes;
  const int BN = wide ? 256 : 128;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[3] = {(uint64_t)p.k, (uint64_t)p.m, (uint64_t)p.batch};
    const uint64_t strides[2] = {(uint64_t)p.a_rstride * 2, (uint64_t)p.a_bstride * 2};
    const uint32_t box[3] = {BK, BM, 1};
    if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.a, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  const int64_t b_rows = p.b_rows > 0 ? p.b_rows : p.n;
  if (p.b_kmajor) {
    const uint64_t dims[3] = {(uint64_t)p.k, (uint64_t)b_rows, (uint64_t)p.batch};
    const uint64_t strides[2] = {(uint64_t)p.b_rstride * 2, (uint64_t)p.b_bstride * 2};
    const uint32_t box[3] = {BK, BN, 1};
    if (!make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.b, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else {
    const uint64_t dims[3] = {(uint64_t)b_rows, (uint64_t)p.k, (uint64_t)p.batch};
    const uint64_t strides[2] = {(uint64_t)p.b_rstride * 2, (uint64_t)p.b_bstride * 2};
    const uint32_t box[3] = {64, BK, 1};
    if (!make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, p.b, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  dim3 grid((unsigned)(p.n / BN), (unsigned)((p.m + BM - 1) / BM), (unsigned)p.batch);
  auto go = [&](auto kern, size_t smem) -> cudaError_t {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem, st>>>(ta, tb, p.b_kmajor, reinterpret_cast<__nv_bfloat16*>(p.c),
                                       p.c_bstride, p.c_rstride, p.m, p.k, qo, rp,
                                       device_error_word());
    return cudaGetLastError();
  };
  if (wide && rp.x) return go(bmm_kernel<2, 256, false, true>, smem_bytes<2, 256>());
  if (rp.x) return cudaErrorInvalidValue;  // the RoPE side comes with the absorb shape only
  if (wide) return go(bmm_kernel<2, 256, false, false>, smem_bytes<2, 256>());
  if (qo.codes) return go(bmm_kernel<4, 128, true, false>, smem_bytes<4, 128>());
  if (p.k / BK <= 2) return go(bmm_kernel<2, 128, false, false>, smem_bytes<2, 128>());
  return go(bmm_kernel<4, 128, false, false>, smem_bytes<4, 128>());
}

}  // namespace qcau
