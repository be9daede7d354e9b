// indexer_score_sm100.cu -- the Lightning Indexer's score rows in one pass
// over the compressed keys (QCAU/QCAU_inference/inference/model.py:518-521,
// Indexer.forward):
//   raw[h, u]   = bf16(q[h, :] . kv[u, :])             the bf16 einsum
//   score[u]    = bf16(sum_h bf16(relu(raw[h, u]) * w[h]))   heads in order
// for each query row (b, s) over the first t keys of its sequence.
//
// The einsum's output ([b, s, h, t] bf16, as large as the keys themselves at
// 64 heads) never reaches memory: the keys are the MMA M (128-key tiles
// streamed by TMA), the query row's heads the N (padded to a multiple of
// 16), so the accumulator holds one key per TMEM lane and its heads along
// the columns, and the epilogue thread of a key sums its heads in order in
// registers.  HBM traffic is the keys once, the queries, and 4 B of score
// per key.
//
// Persistent: one CTA per SM over a contiguous range of (query row, key
// tile) units, 320 threads: warp 0 TMA producer (a ring of key tiles; the
// query row's heads double-buffered), warp 1 TMEM allocator and MMA issuer
// (two accumulators, so a tile's epilogue overlaps the next tile's MMAs),
// warps 2-9 epilogue in two sets of four, one set per accumulator (a
// thread's 64 products and 64 dependent adds take longer than one warp per
// scheduler hides).  Every barrier wait is bounded.
#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kKeys = 128;                   // keys per tile (MMA M)
constexpr int kHalfBytes = kKeys * 64 * 2;   // one 64-dim half of a key tile: 16 KB
constexpr int kTileBytes = 2 * kHalfBytes;   // 128 keys x 128 dims bf16
constexpr int kThreads = 320;  // producer, MMA issuer, 2 x 4 epilogue warps

template <int NPAD>
struct IdxCfg {
  static constexpr int kStages = NPAD >= 128 ? 4 : 5;
  static constexpr int kQHalf = NPAD * 128;  // NPAD heads x 64 dims bf16
  static constexpr int kQBytes = 2 * kQHalf;
  static constexpr uint32_t kTmemCols = 2 * NPAD < 32 ? 32 : 2 * NPAD;
};

template <int kStages>
struct IdxShared {
  uint64_t kfull[kStages], kempty[kStages];
  uint64_t qfull[2], qempty[2];
  uint64_t tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
};

template <int NPAD>
constexpr size_t idx_smem_bytes() {
  using C = IdxCfg<NPAD>;
  return 1024 + (size_t)C::kStages * kTileBytes + 2 * (size_t)C::kQBytes +
         sizeof(IdxShared<C::kStages>);
}

template <int NPAD>
__global__ void __launch_bounds__(kThreads, 1)
    indexer_score_kernel(const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_q,
                         const __nv_bfloat16* __restrict__ w, float* __restrict__ score,
                         int64_t rows, int64_t seqlen, int h, int64_t t, int* err) {
  using C = IdxCfg<NPAD>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* ktiles = smem_raw + pad;
  uint8_t* qbuf = ktiles + (size_t)S * kTileBytes;
  IdxShared<S>* sh = reinterpret_cast<IdxShared<S>*>(qbuf + 2 * (size_t)C::kQBytes);
  volatile int* abort = &sh->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t tiles = (t + kKeys - 1) / kKeys;
  const int64_t units = rows * tiles;
  const int64_t u0 = units * blockIdx.x / gridDim.x;
  const int64_t u1 = units * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&sh->kfull[i], 1);
      mbar_init(&sh->kempty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&sh->qfull[i], 1);
      mbar_init(&sh->qempty[i], 1);
      mbar_init(&sh->tfull[i], 1);
      mbar_init(&sh->tempty[i], 4);
    }
    sh->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<1>(&sh->tmem_base, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------- producer
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_q);
    int last_k[S];
    for (int i = 0; i < S; i++) last_k[i] = -1;
    int last_q[2] = {-1, -1};
    int64_t prev_r = -1;
    int qi = 0;
    for (int64_t u = u0; u < u1; u++) {
      const int64_t r = u / tiles, j = u - r * tiles;
      if (r != prev_r) {
        const int qb = qi & 1, qu = qi >> 1;
        if (!mbar_wait(&sh->qempty[qb], (qu & 1) ^ 1, abort)) break;
        mbar_arrive_expect_tx(&sh->qfull[qb], C::kQBytes);
        uint8_t* qd = qbuf + (size_t)qb * C::kQBytes;
        tma_load_2d(qd, &tm_q, &sh->qfull[qb], 0, (int)(r * h));
        tma_load_2d(qd + C::kQHalf, &tm_q, &sh->qfull[qb], 64, (int)(r * h));
        last_q[qb] = qu;
        qi++;
        prev_r = r;
      }
      const int idx = (int)(u - u0), st = idx % S, us = idx / S;
      if (!mbar_wait(&sh->kempty[st], (us & 1) ^ 1, abort)) break;
      mbar_arrive_expect_tx(&sh->kfull[st], kTileBytes);
      uint8_t* kd = ktiles + (size_t)st * kTileBytes;
      const int seq = (int)(r / seqlen);
      tma_load_3d(kd, &tm_k, &sh->kfull[st], 0, (int)(j * kKeys), seq);
      tma_load_3d(kd + kHalfBytes, &tm_k, &sh->kfull[st], 64, (int)(j * kKeys), seq);
      last_k[st] = us;
    }
    if (*abort) {  // let the copies in flight land before the CTA exits
      volatile int never = 0;
      for (int i = 0; i < S; i++)
        if (last_k[i] >= 0) mbar_wait(&sh->kfull[i], last_k[i] & 1, &never);
      for (int i = 0; i < 2; i++)
        if (last_q[i] >= 0) mbar_wait(&sh->qfull[i], last_q[i] & 1, &never);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = make_idesc(kKeys, NPAD, kFmtBF16, kFmtBF16, false, false);
    int64_t prev_r = -1;
    int qi = 0, last_acc = -1, last_par = 0;
    uint32_t b_base = 0;
    for (int64_t u = u0; u < u1; u++) {
      const int64_t r = u / tiles;
      if (r != prev_r) {
        if (prev_r >= 0) tc_commit(&sh->qempty[(qi - 1) & 1]);
        const int qb = qi & 1, qu = qi >> 1;
        if (!mbar_wait(&sh->qfull[qb], qu & 1, abort)) break;
        b_base = smem_u32(qbuf + (size_t)qb * C::kQBytes);
        qi++;
        prev_r = r;
      }
      const int idx = (int)(u - u0), st = idx % S, us = idx / S;
      const int acc = idx & 1, ua = idx >> 1;
      if (!mbar_wait(&sh->tempty[acc], (ua & 1) ^ 1, abort)) break;
      if (!mbar_wait(&sh->kfull[st], us & 1, abort)) break;
      tc_fence_after();
      const uint32_t a_base = smem_u32(ktiles + (size_t)st * kTileBytes);
      const uint32_t d = tmem + (uint32_t)(acc * NPAD);
#pragma unroll
      for (int half = 0; half < 2; half++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint64_t ad = make_sdesc(a_base + half * kHalfBytes + kk * 32, 16, 1024);
          const uint64_t bd = make_sdesc(b_base + half * C::kQHalf + kk * 32, 16, 1024);
          mma_bf16(d, ad, bd, idesc, (half | kk) ? 1u : 0u);
        }
      tc_commit(&sh->kempty[st]);
      tc_commit(&sh->tfull[acc]);
      last_acc = acc;
      last_par = ua & 1;
    }
    if (*abort && last_acc >= 0) {  // no MMA may still write TMEM when it is freed
      volatile int never = 0;
      mbar_wait(&sh->tfull[last_acc], (uint32_t)last_par, &never);
    }
  } else if (warp >= 2) {
    // ---------------------------------------------------------- epilogue
    // Two sets of four warps, set e taking the units of accumulator e; a
    // warp reads the TMEM lanes of its quarter (warp % 4), one key a thread.
    const int quarter = warp & 3, set = (warp - 2) >> 2;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float wr[NPAD];
    int64_t prev_r = -1;
    for (int64_t u = u0 + set; u < u1; u += 2) {
      const int64_t r = u / tiles, j = u - r * tiles;
      if (r != prev_r) {
        // heads past h (MMA padding) get weight 0: their products are +-0
        // and leave every partial sum as it is
        const __nv_bfloat16* wp = w + r * h;
#pragma unroll
        for (int hh = 0; hh < NPAD; hh++) wr[hh] = hh < h ? __bfloat162float(wp[hh]) : 0.f;
        prev_r = r;
      }
      const int idx = (int)(u - u0), acc = idx & 1, ua = idx >> 1;
      if (!mbar_wait(&sh->tfull[acc], ua & 1, abort)) break;
      tc_fence_after();
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < NPAD / 32 + (NPAD % 32 ? 1 : 0); c++) {
        float v[32];
        if constexpr (NPAD >= 32) {
          tmem_ld32(tmem + lane_addr + (uint32_t)(acc * NPAD + c * 32), v);
          tmem_ld_wait_regs(v);
        } else {
          tmem_ld16(tmem + lane_addr + (uint32_t)(acc * NPAD), *reinterpret_cast<float(*)[16]>(v));
          tmem_ld_wait_regs16(v);
        }
        if (c == (NPAD + 31) / 32 - 1) {  // the accumulator is read: hand it back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh->tempty[acc]);
        }
        constexpr int kCols = NPAD >= 32 ? 32 : 16;
        float p[kCols];
#pragma unroll
        for (int i = 0; i < kCols; i += 2) {
          // raw to bf16 (the einsum's output), ReLU, times the weight, to
          // bf16: two values a conversion
          const float2 rb = __bfloat1622float2(__floats2bfloat162_rn(v[i], v[i + 1]));
          const float m0 = __fmul_rn(fmaxf(rb.x, 0.f), wr[c * 32 + i]);
          const float m1 = __fmul_rn(fmaxf(rb.y, 0.f), wr[c * 32 + i + 1]);
          const float2 pb = __bfloat1622float2(__floats2bfloat162_rn(m0, m1));
          p[i] = pb.x;
          p[i + 1] = pb.y;
        }
#pragma unroll
        for (int i = 0; i < kCols; i++) sum += p[i];  // heads in order
      }
      const int64_t key = j * kKeys + quarter * 32 + lane;
      if (key < t) score[r * t + key] = bf16_round(sum);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(err, QCAU_DEVERR_TIMEOUT);
}

template <int NPAD>
cudaError_t launch_npad(const void* q, const void* kv, const void* w, float* score, int64_t b,
                        int64_t s, int64_t h, int64_t t, int64_t kv_rows, cudaStream_t st) {
  const int64_t rows = b * s;
  CUtensorMap tk, tq;
  {
    const uint64_t dims[3] = {128, (uint64_t)t, (uint64_t)b};
    const uint64_t strides[2] = {256, (uint64_t)kv_rows * 256};
    const uint32_t box[3] = {64, kKeys, 1};
    if (!make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, kv, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[2] = {128, (uint64_t)(rows * h)};
    const uint64_t strides[1] = {256};
    const uint32_t box[2] = {64, (uint32_t)NPAD};
    if (!make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t units = rows * ((t + kKeys - 1) / kKeys);
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  const size_t smem = idx_smem_bytes<NPAD>();
  auto kern = indexer_score_kernel<NPAD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, smem, st>>>(tk, tq, reinterpret_cast<const __nv_bfloat16*>(w), score,
                                     rows, s, (int)h, t, device_error_word());
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_indexer_score_sm100(const void* q, const void* kv, const void* w, float* score,
                                       int64_t b, int64_t s, int64_t h, int64_t t,
                                       int64_t kv_rows, cudaStream_t st) {
  if (b * s == 0 || t == 0) return cudaSuccess;
  if (h <= 0 || h > 128) return cudaErrorInvalidValue;
  if (h <= 16) return launch_npad<16>(q, kv, w, score, b, s, h, t, kv_rows, st);
  if (h <= 32) return launch_npad<32>(q, kv, w, score, b, s, h, t, kv_rows, st);
  if (h <= 64) return launch_npad<64>(q, kv, w, score, b, s, h, t, kv_rows, st);
  return launch_npad<128>(q, kv, w, score, b, s, h, t, kv_rows, st);
}

}  // namespace qcau
