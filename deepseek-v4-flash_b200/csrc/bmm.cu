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
// CTA = one 128 x 128 output tile of one batch entry, 192 threads:
//   warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer,
//   warps 2-5 epilogue (TMEM -> bf16 rows).
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int BM = 128, BN = 128, BK = 64;  // BK bf16 = 128-byte rows
constexpr int kTileBytes = 128 * BK * 2;   // 16 KB
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kThreads = 192;

// Stages of the TMA ring: 2 (66 KB, three CTAs per SM) when K fits in two
// steps, as in the absorb (K = 128); 4 for longer K (the v-up, K = 512).
template <int kStages>
struct BmmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull;
  uint32_t tmem_base;
  int abort;
};
template <int kStages>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)kStages * kStageBytes + sizeof(BmmShared<kStages>);
}

template <int kStages>
__global__ void __launch_bounds__(kThreads, 1)
    bmm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
               int b_kmajor, __nv_bfloat16* __restrict__ c, int64_t c_bstride, int64_t c_rstride,
               int64_t m, int64_t k, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
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
        // two 64-wide N chunks of [64 K rows x 128 B]
        tma_load_3d(st + kTileBytes, &tm_b, &sh->full[s], n0, ks * BK, g);
        tma_load_3d(st + kTileBytes + kTileBytes / 2, &tm_b, &sh->full[s], n0 + 64, ks * BK, g);
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
                                     : make_sdesc(b_addr + kk * 16 * 128, kTileBytes / 2, 1024);
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
    if (mbar_wait(&sh->tfull, 0, abort)) {
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
      __nv_bfloat16* dst = c + g * c_bstride + row * c_rstride + n0;
#pragma unroll
      for (int c4 = 0; c4 < BN / 32; c4++) {
        float v[32];
        tmem_ld32(taddr + c4 * 32, v);
        tmem_ld_wait_regs(v);
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
  if (p.n % BN || p.k % BK) return cudaErrorInvalidValue;
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
                                       p.c_bstride, p.c_rstride, p.m, p.k, device_error_word());
    return cudaGetLastError();
  };
  if (p.k / BK <= 2) return go(bmm_kernel<2>, smem_bytes<2>());
  return go(bmm_kernel<4>, smem_bytes<4>());
}

}  // namespace qcau
