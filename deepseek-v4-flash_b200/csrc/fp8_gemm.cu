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
// CTA = 128 x 128 output tile, 320 threads:
//   warp 0     TMA producer (A and B tiles, 128-byte swizzle, kStages ring)
//   warp 1     TMEM allocator + single-thread MMA issuer
//   warps 2-9  epilogue: TMEM -> registers, scale promotion; two warps per
//              TMEM lane quarter, 64 columns each, so that one 64-column load
//              and one wait per K-block feed 32 packed FMAs
// Four TMEM accumulators (4 x 128 columns) let the MMA run up to three
// K-blocks ahead of the promotion.  The finished tile goes through shared
// memory in the 128-byte swizzled layout (a warp's 16-byte row chunks land in
// distinct banks) and leaves by TMA bulk stores; rows past m are clipped by
// the store.  Split-K partial tiles are parked in padded rows (528 bytes
// apart, conflict-free) and summed over distributed shared memory by 16-byte
// loads, all issued before the first add.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int kStages = 6;
constexpr int kTileBytes = BM * BK;  // fp8: 16 KB per operand tile
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kAcc = 4;              // TMEM accumulators (the MMA runs up to 3 K-blocks ahead)
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter, 64 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kTmemCols = kAcc * BN;
constexpr int64_t kNumSmsGemm = 148;
constexpr int kRedStride = BN + 4;   // floats per row of a parked split-K partial tile
constexpr int kOutTile = 128 * 128;  // bytes of one 128-row x 128-byte output box in smem

struct GemmShared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tfull[kAcc];
  uint64_t tempty[kAcc];
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + sizeof(GemmShared);

__global__ void __launch_bounds__(kThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_c, const void* __restrict__ sa,
                    const void* __restrict__ sb, int64_t m, int64_t k, int a_e8m0, int b_e8m0,
                    int out_f32, int splits, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  GemmShared* sh = reinterpret_cast<GemmShared*>(tiles + (size_t)kStages * kStageBytes);
  volatile int* abort = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n0 = (int64_t)blockIdx.x * BN, m0 = (int64_t)blockIdx.y * BM;
  const int KB = (int)(k / BK);
  // split-K: CTA z of a cluster of `splits` runs K-blocks [kb0, kb1)
  const int z = (int)blockIdx.z;
  const int kb0 = (int)((int64_t)KB * z / splits), kb1 = (int)((int64_t)KB * (z + 1) / splits);
  const int NKB = kb1 - kb0;
  // epilogue role: TMEM lane quarter and 64-column half of the tile
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row_local = quarter * 32 + lane;
  const int64_t row = m0 + row_local;
  uint64_t acc[32];  // epilogue: packed fp32 pairs of this thread's 64 columns
  bool epi_ok = false;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < kAcc; b++) {
      mbar_init(&sh->tfull[b], 1);
      mbar_init(&sh->tempty[b], kEpiWarps);
    }
    sh->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_c);
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
    for (int j = 0; j < NKB; j++) {
      const int kb = kb0 + j;
      const int s = j % kStages;
      const int u = j / kStages;
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
    for (int j = 0; j < NKB; j++) {
      const int s = j % kStages;
      const int u = j / kStages;
      const int ab = j % kAcc;
      const int ua = j / kAcc;
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
      committed = j;
    }
    if (*abort && committed >= 0) {
      // let the issued MMAs finish before TMEM is released
      volatile int never = 0;
      mbar_wait(&sh->tfull[committed % kAcc], (committed / kAcc) & 1, &never);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue: warp w owns TMEM lane quarter w % 4 and the
    // 64 columns [64 * half, +64) of the tile
    const int64_t nblk = n0 / 128;
    // the two scales of K-block kb, loaded kPre blocks ahead: a global load
    // per block would otherwise stall every promotion
    constexpr int kPre = 4;
    auto scale_of = [&](int j) -> float {
      if (j >= NKB) return 0.f;
      const int kb = kb0 + j;
      const float s_a = row < m ? load_scale(sa, row * KB + kb, a_e8m0) : 0.f;
      return s_a * load_scale(sb, nblk * KB + kb, b_e8m0);
    };
    float sc0 = scale_of(0), sc1 = scale_of(1), sc2 = scale_of(2), sc3 = scale_of(3);
#pragma unroll
    for (int i = 0; i < 32; i++) acc[i] = 0ull;
    bool ok = true;
    for (int j = 0; j < NKB; j++) {
      const int ab = j % kAcc;
      const int ua = j / kAcc;
      const float sc = sc0;
      sc0 = sc1;
      sc1 = sc2;
      sc2 = sc3;
      sc3 = scale_of(j + kPre);
      if (!mbar_wait(&sh->tfull[ab], ua & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t sc2x = f2_pack(sc, sc);
      float v[64];
      tmem_ld64(tmem + ((uint32_t)(quarter * 32) << 16) + ab * BN + half * 64, v);
      tmem_ld_wait_regs(v);
      tmem_ld_wait_regs(v + 32);
      // the accumulator may be reused once every epilogue warp has read it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->tempty[ab]);
#pragma unroll
      for (int i = 0; i < 32; i++) acc[i] = f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), sc2x, acc[i]);
    }
    epi_ok = ok;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, kTmemCols);
  }
  __syncwarp();
  if (splits > 1) {
    // the other CTAs of the cluster park their fp32 partial tile in their
    // (now idle) stage buffers; CTA 0 adds them in cluster-rank order
    float* red = reinterpret_cast<float*>(tiles) + row_local * kRedStride + 64 * half;
    if (warp >= 2 && epi_ok && z > 0) {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float a0, a1, a2, a3;
        f2_unpack(acc[2 * i], a0, a1);
        f2_unpack(acc[2 * i + 1], a2, a3);
        reinterpret_cast<float4*>(red)[i] = make_float4(a0, a1, a2, a3);
      }
    }
    cluster_sync();
    if (warp >= 2 && epi_ok && z == 0) {
      for (int zz = 1; zz < splits; zz++) {
        const uint32_t src = mapa_shared(smem_u32(red), (uint32_t)zz);
        float4 r[16];
#pragma unroll
        for (int i = 0; i < 16; i++) r[i] = ld_shared_cluster_v4f32(src + 16 * i);
#pragma unroll
        for (int i = 0; i < 16; i++) {
          acc[2 * i] = f2_add(acc[2 * i], f2_pack(r[i].x, r[i].y));
          acc[2 * i + 1] = f2_add(acc[2 * i + 1], f2_pack(r[i].z, r[i].w));
        }
      }
    }
    cluster_sync();
  }
  if (warp >= 2 && z == 0) {
    // the tile into swizzled 128-row x 128-byte boxes: bf16 -> box `half`
    // (64 columns), fp32 -> boxes 2 * half, 2 * half + 1 (32 columns each);
    // 16-byte chunk j of row r sits at r * 128 + ((j ^ (r & 7)) * 16)
    float out[64];
#pragma unroll
    for (int i = 0; i < 32; i++) f2_unpack(acc[i], out[2 * i], out[2 * i + 1]);
    const int sw = row_local & 7;
    if (out_f32) {
#pragma unroll
      for (int q = 0; q < 2; q++) {
        uint8_t* box = tiles + (size_t)(2 * half + q) * kOutTile + row_local * 128;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float* v = out + 32 * q + 4 * j;
          *reinterpret_cast<float4*>(box + ((j ^ sw) << 4)) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    } else {
      uint8_t* box = tiles + (size_t)half * kOutTile + row_local * 128;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(out[8 * j + 0], out[8 * j + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(out[8 * j + 2], out[8 * j + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(out[8 * j + 4], out[8 * j + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(out[8 * j + 6], out[8 * j + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(box + ((j ^ sw) << 4)) = pk;
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 32 * kEpiWarps);
    if (warp == 2 && lane == 0 && !*abort) {
      if (out_f32) {
        for (int t = 0; t < 4; t++) tma_store_2d(&tm_c, tiles + (size_t)t * kOutTile, (int)n0 + 32 * t, (int)m0);
      } else {
        for (int t = 0; t < 2; t++) tma_store_2d(&tm_c, tiles + (size_t)t * kOutTile, (int)n0 + 64 * t, (int)m0);
      }
      bulk_commit_group();
      bulk_wait_group0();
    }
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(err, QCAU_DEVERR_TIMEOUT);
}

}  // namespace

cudaError_t launch_fp8_gemm(const void* a, const void* a_s, const void* b, const void* b_s,
                            void* c, int64_t m, int64_t n, int64_t k, int a_e8m0, int b_e8m0,
                            int out_f32, cudaStream_t st) {
  if (m == 0) return cudaSuccess;
  if (n % BN || k % BK) return cudaErrorInvalidValue;
  CUtensorMap ta, tb, tc;
  const uint64_t da[2] = {(uint64_t)k, (uint64_t)m};
  const uint64_t db[2] = {(uint64_t)k, (uint64_t)n};
  const uint64_t sa_[1] = {(uint64_t)k};
  const uint32_t box[2] = {BK, BM};
  // C as [m][n] of 2- or 4-byte values, stored in 128-byte-wide boxes
  const uint64_t dc[2] = {(uint64_t)n, (uint64_t)m};
  const uint64_t sc_[1] = {(uint64_t)n * (out_f32 ? 4 : 2)};
  const uint32_t cbox[2] = {out_f32 ? 32u : 64u, (uint32_t)BM};
  if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, da, sa_, box,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, b, db, sa_, box,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap(&tc, out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                 c, dc, sc_, cbox, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  // few output tiles (decode-size m): split K over a cluster so that every SM
  // streams weights; the partial tiles are summed through distributed shared
  // memory, in a fixed order
  const int64_t tiles = (n / BN) * ((m + BM - 1) / BM);
  const int64_t kblocks = k / BK;
  int splits = 1;
  if (tiles * 4 <= kNumSmsGemm && kblocks >= 16) splits = 4;
  else if (tiles * 2 <= kNumSmsGemm && kblocks >= 8) splits = 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n / BN), (unsigned)((m + BM - 1) / BM), (unsigned)splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)splits;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fp8_gemm_kernel, ta, tb, tc, a_s, b_s, m, k, a_e8m0, b_e8m0,
                            out_f32, splits, device_error_word());
}

}  // namespace qcau
