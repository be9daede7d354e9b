// fp8_gemm.cu -- FP8 e4m3 block-scaled GEMM on the sm_100a tensor cores.
//
// Replaces kernel.fp8_gemm (Deepseek_origin/inference/kernel.py:257-273,
// TileLang kernel :203-254; C++ port qcau_c/src/qcau.cpp:30-90):
//   C[m, n] = sum_kb (A[m, kb] . B[n, kb]) * sa[m, kb] * sb[n / 128, kb]
// with the reference's two-level accumulation: every 128-wide K block is
// accumulated in fp32 by tcgen05.mma (kind::f8f6f4) into a TMEM buffer and
// then promoted with its two scales into a register accumulator
// (kernel.py:246-250).  Scales may be fp32 or E8M0.
//
// CTA = 128 x 128 output tile, 192 threads:
//   warp 0     TMA producer (A and B tiles, 128-byte swizzle, kStages ring)
//   warp 1     TMEM allocator + single-thread MMA issuer
//   warps 2-5  epilogue: TMEM -> registers, scale promotion, bf16/fp32 store
// Two TMEM accumulators (2 x 128 columns) let the MMA of block kb+1 run
// while the epilogue promotes block kb.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int kStages = 6;
constexpr int kTileBytes = BM * BK;  // fp8: 16 KB per operand tile
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kThreads = 192;
constexpr int kTmemCols = 2 * BN;

struct GemmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + sizeof(GemmShared);

__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const void* __restrict__ sa, const void* __restrict__ sb, void* __restrict__ c,
                    int64_t m, int64_t n, int64_t k, int a_e8m0, int b_e8m0, int out_f32, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  GemmShared* sh = reinterpret_cast<GemmShared*>(tiles + (size_t)kStages * kStageBytes);
  volatile int* abort = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * BN, m0 = (int64_t)blockIdx.y * BM;
  const int KB = (int)(k / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&sh->tfull[b], 1);
      mbar_init(&sh->tempty[b], 4);
    }
    sh->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) tmem_alloc<1>(&sh->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    int last_use[kStages];
    for (int s = 0; s < kStages; s++) last_use[s] = -1;
    for (int kb = 0; kb < KB; kb++) {
      const int s = kb % kStages;
      const int u = kb / kStages;
      if (!mbar_wait(&sh->empty[s], (u & 1) ^ 1, abort)) break;
      mbar_arrive_expect_tx(&sh->full[s], kStageBytes);
      uint8_t* st = tiles + (size_t)s * kStageBytes;
      tma_load_2d(st, &tm_a, &sh->full[s], kb * BK, (int)m0);
      tma_load_2d(st + kTileBytes, &tm_b, &sh->full[s], kb * BK, (int)n0);
      last_use[s] = u;
    }
    if (*abort) {
      // drain this CTA's copies still in flight before the CTA exits
      volatile int never = 0;
      for (int s = 0; s < kStages; s++)
        if (last_use[s] >= 0) mbar_wait(&sh->full[s], last_use[s] & 1, &never);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t idesc = make_idesc(BM, BN, kFmtE4M3, kFmtE4M3, false, false);
    int committed = -1;
    for (int kb = 0; kb < KB; kb++) {
      const int s = kb % kStages;
      const int u = kb / kStages;
      const int ab = kb & 1;
      const int ua = kb >> 1;
      if (!mbar_wait(&sh->full[s], u & 1, abort)) break;
      if (!mbar_wait(&sh->tempty[ab], (ua & 1) ^ 1, abort)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(tiles + (size_t)s * kStageBytes);
      const uint32_t b_addr = a_addr + kTileBytes;
#pragma unroll
      for (int kk = 0; kk < BK / 32; kk++) {
        const uint64_t ad = make_sdesc(a_addr + kk * 32, 16, 1024);
        const uint64_t bd = make_sdesc(b_addr + kk * 32, 16, 1024);
        mma_f8f6f4(tmem + ab * BN, ad, bd, idesc, kk > 0 ? 1u : 0u);
      }
      tc_commit(&sh->empty[s]);
      tc_commit(&sh->tfull[ab]);
      committed = kb;
    }
    if (*abort && committed >= 0) {
      // let the issued MMAs finish before TMEM is released
      volatile int never = 0;
      mbar_wait(&sh->tfull[committed & 1], (committed >> 1) & 1, &never);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_local = quarter * 32 + lane;
    const int64_t row = m0 + row_local;
    const int64_t nblk = n0 / 128;
    // the two scales of K-block kb, loaded kPre blocks ahead: a global load
    // per block would otherwise stall every promotion
    constexpr int kPre = 4;
    auto scale_of = [&](int kb) -> float {
      if (kb >= KB) return 0.f;
      const float s_a = row < m ? load_scale(sa, row * KB + kb, a_e8m0) : 0.f;
      return s_a * load_scale(sb, nblk * KB + kb, b_e8m0);
    };
    float sc0 = scale_of(0), sc1 = scale_of(1), sc2 = scale_of(2), sc3 = scale_of(3);
    uint64_t acc[BN / 2];  // packed fp32 pairs
#pragma unroll
    for (int i = 0; i < BN / 2; i++) acc[i] = 0ull;
    bool ok = true;
    for (int kb = 0; kb < KB; kb++) {
      const int ab = kb & 1;
      const int ua = kb >> 1;
      const float sc = sc0;
      sc0 = sc1;
      sc1 = sc2;
      sc2 = sc3;
      sc3 = scale_of(kb + kPre);
      if (!mbar_wait(&sh->tfull[ab], ua & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t sc2x = f2_pack(sc, sc);
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + ab * BN;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float v[64];
        tmem_ld32(taddr + h * 64, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld32(taddr + h * 64 + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        tmem_ld_wait_regs(v);
        tmem_ld_wait_regs(v + 32);
#pragma unroll
        for (int i = 0; i < 32; i++)
          acc[h * 32 + i] = f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), sc2x, acc[h * 32 + i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->tempty[ab]);
    }
    if (ok && row < m) {
      float out[BN];
#pragma unroll
      for (int i = 0; i < BN / 2; i++) f2_unpack(acc[i], out[2 * i], out[2 * i + 1]);
      if (out_f32) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(c) + row * n + n0);
#pragma unroll
        for (int j = 0; j < BN / 4; j++)
          dst[j] = make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(c) + row * n + n0);
#pragma unroll
        for (int j = 0; j < BN / 8; j++) {
          uint4 pk;
          __nv_bfloat162 h0 = __floats2bfloat162_rn(out[8 * j + 0], out[8 * j + 1]);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(out[8 * j + 2], out[8 * j + 3]);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(out[8 * j + 4], out[8 * j + 5]);
          __nv_bfloat162 h3 = __floats2bfloat162_rn(out[8 * j + 6], out[8 * j + 7]);
          pk.x = *reinterpret_cast<uint32_t*>(&h0);
          pk.y = *reinterpret_cast<uint32_t*>(&h1);
          pk.z = *reinterpret_cast<uint32_t*>(&h2);
          pk.w = *reinterpret_cast<uint32_t*>(&h3);
          dst[j] = pk;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(err, QCAU_DEVERR_TIMEOUT);
}

}  // namespace

cudaError_t launch_fp8_gemm(const void* a, const void* a_s, const void* b, const void* b_s,
                            void* c, int64_t m, int64_t n, int64_t k, int a_e8m0, int b_e8m0,
                            int out_f32, cudaStream_t st) {
  if (m == 0) return cudaSuccess;
  CUtensorMap ta, tb;
  const uint64_t da[2] = {(uint64_t)k, (uint64_t)m};
  const uint64_t db[2] = {(uint64_t)k, (uint64_t)n};
  const uint64_t sa_[1] = {(uint64_t)k};
  const uint32_t box[2] = {BK, BM};
  if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, da, sa_, box,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, db, sa_, box,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)(n / BN), (unsigned)((m + BM - 1) / BM));
  fp8_gemm_kernel<<<grid, kThreads, kSmemBytes, st>>>(ta, tb, a_s, b_s, c, m, n, k, a_e8m0,
                                                      b_e8m0, out_f32, device_error_word());
  return cudaGetLastError();
}

}  // namespace qcau
