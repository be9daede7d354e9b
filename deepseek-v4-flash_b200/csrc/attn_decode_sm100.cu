// attn_decode_sm100.cu -- tcgen05 two-CTA split-KV decode attention over a
// paged latent cache (absorbed MLA: 576-wide K rows, V = first 512 values).
//
// Numerics are those of the reference attention core
// (Deepseek_origin/inference/kernel.py:276-352): fp32 scores, online softmax,
// P rounded to bf16 before P.V, denominator summed from fp32 P; the sink and
// the final normalisation are applied by attn_combine (kernel.py:345-348).
// The running max is the reference's: every tile that raises it rescales O
// (in TMEM) and the denominator, so P is rounded to bf16 at the exact running
// max and the tile's largest score gets P = 1 exactly, as kernel.py:331-343
// computes.  (A stale max, raised only beyond a threshold, saves the O
// rescales but rounds the dominant tokens' P at another scale; at 2^8 that
// moved outputs of near-full-length rows up to 1 % from the reference.)  The
// tile is 128 tokens where the reference's is 64: the max of the whole tile
// scales both pages' P.
//
// Work unit = one sequence x one KV split x 128 heads, run by one CTA pair
// (cluster of 2); tiles of 128 tokens (2 pages).  When the units outnumber the
// pairs that fit on the device, the grid is one pair per slot and each pair
// runs units pair, pair + npairs, ...: TMEM, the barriers and the launch are
// paid once, the next unit's Q loads as soon as the last QK of the current
// one has completed, and its QK tiles run under the current epilogue.  CTA r of the pair owns heads
// [64r, 64r+64) of the group.  With h = 64, 32 or 16 heads (a head shard of
// 128) the pair owns all h heads, h/2 per CTA, and the remaining MMA rows of
// each CTA are padding (Q rows of other heads, or zeros past h) whose outputs
// are not written: the cache bytes, which bound the kernel, are the same.
//   QK : tcgen05.mma.cta_group::2, M = 128 heads, N = 128 tokens (CTA r
//        supplies page 2t+r), K = 576 in 9 chunks of 64
//        -> S in TMEM, 2x2 lane layout: lanes 0-63 tokens 0-63, lanes
//        64-127 tokens 64-127 of the CTA's 64 heads (64 columns, two buffers)
//   PV : cta_group::2, M = 128 heads, N = 256 dims (two MMAs cover 512),
//        K = 128 tokens; A = bf16 P in shared memory, B = V rows given
//        MN-major (for MMA j, CTA r supplies dims [256r + 128j, +128))
//        -> O in TMEM, MMA j at columns [128j, +128): lanes 0-63 dims
//        [128j, +128), lanes 64-127 dims [256 + 128j, +128)
// Issue-rate notes (measured on B200): pair MMAs with N = 128 run at two
// thirds of the rate of N = 256; a blocking mbarrier wait in the issuing
// thread costs hundreds of cycles even when the phase is complete, and the
// tensor queue is shallow, so QK and PV are issued by two different threads
// (one stream's waits are covered by the other's queued MMAs), every wait
// guards at least 8 MMAs, and TMA barriers are waited with CTA scope and no
// tcgen05 fence per chunk.
// Shared memory: Q (64 heads x 576, 72 KB), P (64 heads x 128 tokens, 16 KB),
// a K ring of 3 x 24 KB slots (three 64-dim chunks of the CTA's page) and a
// V ring of 2 x 32 KB slots (one page x the CTA's 256 dims), each ring with
// its own producer warp.  The TMA engine's cost is per box (8 KB boxes of
// 128-byte rows cap a CTA at ~32 GB/s, 24-32 KB boxes reach HBM bandwidth),
// so K and V come in multi-chunk boxes of one page from a 4-D view of the
// cache [pages][64 tokens][9 chunks][64 values]; the 128-token tile is what
// lets each CTA's QK operand be a single page.  A bulk L2 prefetch of whole
// pages ahead of the K reads was measured to add DRAM reads and to cost ~20%
// of the time: none.
// Warps: 0 K producer, 1 TMEM allocator + QK issuer (pair leader), 2-5
// softmax / O correction / epilogue (one TMEM lane each), 6 V producer,
// 7 PV issuer (pair leader).
// Every wait is bounded; a timeout raises QCAU_DEVERR_TIMEOUT, drains the
// copies in flight, frees TMEM and returns.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace qcau {
namespace {

constexpr int kThreads = 256;
constexpr int kTile = 128;            // tokens per tile (two pages, one per CTA for K)
constexpr int kKSlot = 24576;         // this CTA's page x 3 chunks of 64 dims (one box)
constexpr int kKSlots = 3;
constexpr int kKPerTile = 3;          // 9 chunks = 576 dims in 3 boxes
constexpr int kVSlot = 32768;         // one page x this CTA's 256 dims (4 chunks, one box)
constexpr int kVSlots = 2;
constexpr int kVPerTile = 2;          // the tile's 2 pages
constexpr int kQBytes = 9 * 8192;     // 64 heads x 576 bf16 (9 chunks of 64 rows)
constexpr int kPBytes = 2 * 8192;     // 64 heads x 128 tokens bf16 (2 chunks of 64 tokens)
constexpr float kLog2e = 1.4426950408889634f;
// The running max (log2 units) is raised when a tile's max exceeds it by more
// than kRescale; 0 is the reference's exact running max per tile.
#ifndef QCAU_DECODE_RESCALE_LOG2
#define QCAU_DECODE_RESCALE_LOG2 0.0f
#endif
constexpr float kRescale = QCAU_DECODE_RESCALE_LOG2;

constexpr uint32_t kTmemO = 0;        // 2 accumulators x 128 columns
constexpr uint32_t kTmemS = 256;      // 2 buffers x 64 columns
constexpr uint32_t kTmemCols = 512;

struct DecodeShared {
  uint64_t kfull[kKSlots];   // leader: K slot landed in both CTAs
  uint64_t kempty[kKSlots];  // both: K slot consumed by QK (the last slot: s_full)
  uint64_t vfull[kVSlots];   // leader: V slot landed in both CTAs
  uint64_t vempty[kVSlots];  // both: V slot consumed by PV (the last slot: p_free)
  uint64_t q_full;           // leader: Q landed in both CTAs
  uint64_t s_full[2];        // both: S(t) ready
  uint64_t s_free[2];        // leader: the 8 softmax warps have read S(t)
  uint64_t p_full;           // leader: the 8 softmax warps wrote P(t) / corrected O
  uint64_t p_free;           // both: PV(t) done with P and O
  uint64_t o_full;           // both: last PV of the unit done
  uint64_t q_empty;          // both: last QK of the unit done (Q may be reloaded)
  uint64_t o_free;           // leader: the 8 epilogue warps have read O
  uint64_t xbar[2];          // local: the 4 softmax warps exchanged tile maxima
  uint64_t lbar;             // local: denominator exchange
  float xmax[2][128];
  float xsum[128];
  uint32_t tmem_base;
  int abort;
  long long tiles[8];  // per warp: the batch's tiles (the balanced schedule's check)
};

static_assert(kKSlots == kKPerTile && kVSlots == kVPerTile,
              "each ring holds exactly one tile: slot i is box i of the tile");

constexpr size_t kSmemBytes = 1024 + kQBytes + kPBytes + (size_t)kKSlots * kKSlot +
                              (size_t)kVSlots * kVSlot + sizeof(DecodeShared);
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr int kMaxBlocks = 16;  // destination head blocks of the partials

struct DecodeParams {
  const int32_t* table;
  const int32_t* seqlens;
  __nv_bfloat16* out;  // direct mode (one split): final output [rows, h, 512]
  const float* sink;   // direct mode: attention sink [h] or nullptr
  int* err;
  int64_t max_pages, num_pages;
  int h, hgroups, splits;
  int cta_heads;  // heads each CTA owns: 64, or h/2 when h < 128 (the other MMA rows are padding)
  float scale;
  int qlen;    // query tokens per sequence (1 = decode; > 1 = causal prefill / chunk)
  int direct;  // 1: one split, the epilogue normalises and writes `out`
  // context-parallel decode over ranks: Q boxes of q_box heads from blocks of
  // q_hblock heads; splits [split_base, +splits) of splits_total; the
  // partials of head block j (part_hblock heads) go to blk_o[j] / blk_ml[j],
  // [rows][splits][part_hblock] each: local blocks, or the receive slots of
  // the ranks that own the heads (peer memory over NVLink)
  int q_hblock, q_box;
  int split_base, splits_total;
  int part_hblock;
  int nblk;
  int o_hblock;   // direct mode: o as [h / o_hblock][rows][o_hblock][512]
  int64_t rows;
  int64_t units;  // work units; pair i of the grid runs units i, i + pairs, ...
  // balanced schedule (stream != 0, one query token per sequence): pair i
  // runs tiles [i G / pairs, (i + 1) G / pairs) of the G = rows x hgroups x
  // nt tiles, row after row; a row's pieces fill its partial slots in pair
  // order, and its last piece marks the slots after it empty.  It is taken
  // when the sequences fill at least 90 % of the rows x nt tiles; otherwise
  // the same launch runs `splits` equal splits of each row's own tiles,
  // units looped over the pairs
  int stream;
  int64_t nt, gtiles;
  int usplits;  // equal splits of a row in the unit enumeration (<= splits, the partial slots)
  void* blk_o[kMaxBlocks];     // fp32 O, or fp16 O / l when part_f16
  int part_f16;
  float* blk_ml[kMaxBlocks];
  // completion: when `counter` is set, the last CTA to finish raises
  // flag[j] = epoch (release, system scope) for every block destination j
  uint32_t* flag[kMaxBlocks];
  unsigned int* counter;
  uint32_t epoch;
};

// Called by thread 0 of each CTA once all the CTA's partial stores are
// ordered before it (a CTA or cluster barrier): counts the CTA, and the last
// one of the grid publishes `epoch` to every destination's flag.
__device__ __forceinline__ void signal_done(const DecodeParams& p) {
  if (p.counter == nullptr) return;
  __threadfence_system();
  unsigned int prev;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
               : "=r"(prev)
               : "l"(p.counter)
               : "memory");
  if (prev == gridDim.x - 1) {
    __threadfence_system();
    for (int j = 0; j < p.nblk; j++)
      asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flag[j]), "r"(p.epoch) : "memory");
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p.counter), "r"(0u) : "memory");
  }
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One work unit: query row b (sequence bs), KV split, and the first head of
// this CTA's half of the 128-head group.
struct DecodeUnit {
  int64_t b, bs;
  int split, seqlen, t_begin, T, head0;
  int empty_from;  // partial slots [empty_from, splits) of row b are marked empty
};

__device__ __forceinline__ DecodeUnit decode_unit(const DecodeParams& p, int64_t unit,
                                                  uint32_t rank) {
  DecodeUnit U;
  const int hg = (int)(unit % p.hgroups);
  const int64_t rest = unit / p.hgroups;
  U.split = (int)(rest % p.usplits);
  // query row r = (sequence bs, token t of qlen): token t sees the cached
  // prefix up to its own position, seqlens[bs] - (qlen - 1 - t) tokens
  U.b = rest / p.usplits;
  U.bs = U.b / p.qlen;
  U.seqlen = p.seqlens[U.bs] - (p.qlen - 1 - (int)(U.b % p.qlen));
  const int ntiles = (U.seqlen + kTile - 1) / kTile;
  const int gsplit = p.split_base + U.split;  // this split among splits_total
  U.t_begin = (int)((int64_t)ntiles * gsplit / p.splits_total);
  const int t_end = (int)((int64_t)ntiles * (gsplit + 1) / p.splits_total);
  U.T = t_end - U.t_begin;
  U.head0 = hg * 2 * p.cta_heads + (int)rank * p.cta_heads;
  U.empty_from = p.usplits;  // the balanced schedule's fall-back leaves slots past usplits empty
  return U;
}

// Balanced schedule: the piece of (row, head group) v = g / nt that starts
// at global tile g and ends at g_end or at the row's end.  Its partial slot
// is its pair's rank among the pairs that cover the row; the pair covering
// tile x is the largest q with floor(q G / P) <= x.
__device__ __forceinline__ DecodeUnit stream_unit(const DecodeParams& p, int64_t g, int64_t g_end,
                                                  int64_t pair, int64_t npairs, uint32_t rank) {
  DecodeUnit U;
  const int64_t v = g / p.nt;
  const int hg = (int)(v % p.hgroups);
  U.b = v / p.hgroups;
  U.bs = U.b;
  U.seqlen = p.seqlens[U.bs];
  // the schedule covers max_len tokens a row: a longer sequence is cut there
  if (U.seqlen > p.nt * kTile) raise_dev_error(p.err, QCAU_DEVERR_INDEX);
  const int64_t row0 = v * p.nt, row1 = row0 + p.nt;
  const int64_t first_pair = ((row0 + 1) * npairs - 1) / p.gtiles;
  U.split = (int)(pair - first_pair);
  U.t_begin = (int)(g - row0);
  const int t_end = (int)((g_end < row1 ? g_end : row1) - row0);
  const int ntiles = (U.seqlen + kTile - 1) / kTile;
  U.T = (t_end < ntiles ? t_end : ntiles) - U.t_begin;
  U.head0 = hg * 2 * p.cta_heads + (int)rank * p.cta_heads;
  U.empty_from = row1 <= g_end ? U.split + 1 : p.splits;
  return U;
}

// A pair's walk over its work: units pair, pair + npairs, ... or, in the
// balanced schedule, the pieces of its tile range.  Every role of the pair
// takes the same walk.
struct UnitCursor {
  int64_t pos, end;
};

__device__ __forceinline__ UnitCursor cursor_begin(const DecodeParams& p, bool balanced,
                                                   int64_t pair, int64_t npairs) {
  if (balanced) return {pair * p.gtiles / npairs, (pair + 1) * p.gtiles / npairs};
  return {pair, p.units};
}

__device__ __forceinline__ DecodeUnit cursor_unit(const DecodeParams& p, bool balanced,
                                                  const UnitCursor& c, int64_t pair,
                                                  int64_t npairs, uint32_t rank) {
  return balanced ? stream_unit(p, c.pos, c.end, pair, npairs, rank) : decode_unit(p, c.pos, rank);
}

__device__ __forceinline__ void cursor_next(const DecodeParams& p, bool balanced, UnitCursor& c,
                                            int64_t npairs) {
  c.pos = balanced ? (c.pos / p.nt + 1) * p.nt : c.pos + npairs;
}

// All lanes wait; the warp agrees on the outcome (timeouts are per lane).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait<true>(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    decode_attn_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* sQ = smem_raw + pad;
  uint8_t* sP = sQ + kQBytes;
  uint8_t* sK = sP + kPBytes;
  uint8_t* sV = sK + (size_t)kKSlots * kKSlot;
  DecodeShared* sh = reinterpret_cast<DecodeShared*>(sV + (size_t)kVSlots * kVSlot);
  volatile int* abort = &sh->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  // partial row of (row b, split slot, head) in its head block's destination
  auto part_row_at = [&](int64_t b, int slot, int head, int& blk) -> int64_t {
    blk = head / p.part_hblock;
    return ((int64_t)b * p.splits + slot) * p.part_hblock + (head - blk * p.part_hblock);
  };
  auto part_row = [&](const DecodeUnit& U, int head, int& blk) -> int64_t {
    return part_row_at(U.b, U.split, head, blk);
  };

  // direct-mode output row of (row U.b, head)
  auto out_row = [&](const DecodeUnit& U, int head) -> __nv_bfloat16* {
    const int blk = head / p.o_hblock;
    return p.out + (((int64_t)blk * p.rows + U.b) * p.o_hblock + (head - blk * p.o_hblock)) * 512;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kKSlots; i++) {
      mbar_init(&sh->kfull[i], 1);
      mbar_init(&sh->kempty[i], 1);
    }
    for (int i = 0; i < kVSlots; i++) {
      mbar_init(&sh->vfull[i], 1);
      mbar_init(&sh->vempty[i], 1);
    }
    mbar_init(&sh->q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(&sh->s_full[i], 1);
      mbar_init(&sh->s_free[i], 8);
      mbar_init(&sh->xbar[i], 4);
    }
    mbar_init(&sh->p_full, 8);
    mbar_init(&sh->p_free, 1);
    mbar_init(&sh->o_full, 1);
    mbar_init(&sh->q_empty, 1);
    mbar_init(&sh->o_free, 8);
    mbar_init(&sh->lbar, 4);
    sh->abort = 0;
    fence_barrier_init();
  }
  if (p.stream) {
    // the batch's tiles at its own lengths, to check that it fills the
    // balanced plan (every CTA counts the same, so all take one schedule)
    long long n = 0;
    for (int64_t r = threadIdx.x; r < p.rows; r += kThreads) {
      const int64_t t = ((int64_t)p.seqlens[r] + kTile - 1) / kTile;
      n += t < 0 ? 0 : (t > p.nt ? p.nt : t);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n += __shfl_down_sync(0xffffffffu, n, o);
    if (lane == 0) sh->tiles[warp] = n;
  }
  if (warp == 1) tmem_alloc<2>(&sh->tmem_base, kTmemCols);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  bool balanced = false;
  if (p.stream) {
    long long n = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; w++) n += sh->tiles[w];
    balanced = n * 10 >= (long long)p.rows * p.nt * 9;
  }

  // physical page of the unit's page pidx (units with T > 0 have seqlen >= 1)
  auto page_of = [&](const DecodeUnit& U, int pidx) -> int {
    const int pages_used = (U.seqlen + 63) / 64;
    if (pidx >= pages_used) pidx = pages_used - 1;  // masked tokens: any valid page
    const int64_t e = p.table[U.bs * p.max_pages + pidx];
    if (e < 0 || e >= p.num_pages) {
      raise_dev_error(p.err, QCAU_DEVERR_INDEX);
      return 0;
    }
    return (int)e;
  };

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------ TMA producers (both CTAs)
    // warp 0: per unit Q, then the K boxes of its tiles; warp 6: the V pages.
    if (lane == 0) {
      const bool is_k = warp == 0;
      uint64_t* fullb = is_k ? sh->kfull : sh->vfull;
      uint64_t* emptyb = is_k ? sh->kempty : sh->vempty;
      const int nslots = is_k ? kKSlots : kVSlots;
      const int per_tile = is_k ? kKPerTile : kVPerTile;
      constexpr int kMaxSlots = kKSlots > kVSlots ? kKSlots : kVSlots;
      int last_use[kMaxSlots];  // per slot: last ring pass whose copy was issued
      for (int i = 0; i < kMaxSlots; i++) last_use[i] = -1;
      const uint32_t q_full_l = mapa_shared(smem_u32(&sh->q_full), 0);
      int n = 0, nq = 0;  // ring copies issued; units whose Q was issued
      bool ok = true;
      for (UnitCursor c = cursor_begin(p, balanced, pair, npairs); c.pos < c.end && ok;
           cursor_next(p, balanced, c, npairs)) {
        const DecodeUnit U = cursor_unit(p, balanced, c, pair, npairs, rank);
        if (U.T <= 0) continue;
        if (is_k) {
          // Q of the previous unit is free once its last QK has completed
          if (nq > 0 && !(ok = mbar_wait(&sh->q_empty, (nq - 1) & 1, abort))) break;
          if (leader) mbar_arrive_expect_tx(&sh->q_full, 2 * kQBytes);
          // 64 head rows per chunk, in boxes of q_box heads of one block
          // (rows past the last head are zero-filled padding)
          for (int k = 0; k < 9; k++)
            for (int m = 0; m < 64; m += p.q_box) {
              const int hd = U.head0 + m;
              tma_load_4d_pair(sQ + k * 8192 + m * 128, &tm_q, q_full_l, 64 * k,
                               hd % p.q_hblock, (int)U.b, hd / p.q_hblock);
            }
          nq++;
        }
        for (int it = 0; it < U.T && ok; it++) {
          const int t = U.t_begin + it;
          for (int i = 0; i < per_tile; i++, n++) {
            // slot i of the ring holds box i of a tile (u = the tile's ordinal)
            const int slot = n % nslots, u = n / nslots;
            // the tile's last box is released by the tile's completion commit
            // (QK: s_full, PV: p_free); the others by their own empty barrier
            if (slot == nslots - 1) {
              if (u > 0 && !(ok = is_k ? mbar_wait(&sh->s_full[(u - 1) & 1], ((u - 1) >> 1) & 1, abort)
                                       : mbar_wait(&sh->p_free, (u - 1) & 1, abort)))
                break;
            } else if (!(ok = mbar_wait(&emptyb[slot], (u & 1) ^ 1, abort))) {
              break;
            }
            if (leader) mbar_arrive_expect_tx(&fullb[slot], is_k ? 2 * kKSlot : 2 * kVSlot);
            last_use[slot] = u;
            const uint32_t fb = mapa_shared(smem_u32(&fullb[slot]), 0);
            if (is_k) {
              // chunks 3i..3i+2 (dims 192i..192i+191) of this CTA's page of the tile
              tma_load_4d_pair(sK + slot * kKSlot, &tm_k, fb, 0, 0, 3 * i,
                               page_of(U, 2 * t + (int)rank));
            } else {
              // page i of the tile: this CTA's dims [256r, 256r+256), 4 chunks in one box
              tma_load_4d_pair(sV + slot * kVSlot, &tm_v, fb, 0, 0, 4 * (int)rank,
                               page_of(U, 2 * t + i));
            }
          }
        }
      }
      if (*abort && leader) {
        // the leader's full barriers count both CTAs' copies: drain them all
        volatile int never = 0;
        if (is_k && nq > 0) mbar_wait<true>(&sh->q_full, (nq - 1) & 1, &never);
        for (int slot = 0; slot < nslots; slot++)
          if (last_use[slot] >= 0) mbar_wait<true>(&fullb[slot], last_use[slot] & 1, &never);
      }
    }
  } else if (warp == 1 || warp == 7) {
    // ------------------------------------------------ MMA issuers (pair leader)
    // warp 1 issues QK(0), QK(1), ...; warp 7 issues PV(0), PV(1), ... over
    // the pair's tiles in unit order (gt counts them across units)
    if (leader && lane == 0) {
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      uint64_t* last_bar = nullptr;  // barrier of the last commit, for the drain
      int last_phase = 0;
      bool ok = true;
      if (warp == 1) {
        const uint32_t idesc_qk = make_idesc(128, 128, kFmtBF16, kFmtBF16, false, false);
        const uint64_t q_desc = make_sdesc(q_addr, 16, 1024), k_desc = make_sdesc(k_addr, 16, 1024);
        int nk = 0, gt = 0, nu = 0;  // K boxes consumed, tiles, units
        for (UnitCursor c = cursor_begin(p, balanced, pair, npairs); c.pos < c.end && ok;
             cursor_next(p, balanced, c, npairs)) {
          const DecodeUnit U = cursor_unit(p, balanced, c, pair, npairs, rank);
          if (U.T <= 0) continue;
          if (!(ok = mbar_wait(&sh->q_full, nu & 1, abort))) break;
          for (int it = 0; it < U.T && ok; it++, gt++) {
            const int sb = gt & 1;
            if (gt >= 2 && !(ok = mbar_wait<true>(&sh->s_free[sb], ((gt >> 1) - 1) & 1, abort)))
              break;
            tc_fence_after();
            for (int g = 0; g < kKPerTile; g++, nk++) {
              const int slot = g, u = gt;  // the ring holds one tile: box g in slot g
              if (!(ok = mbar_wait(&sh->kfull[slot], u & 1, abort))) break;
              // chunk k = 3g + c: 4 MMAs of 16 dims, B = this CTA's 64 tokens (N = 128);
              // descriptors advance by (byte offset >> 4) in their address field
              const uint64_t qg = q_desc + (uint64_t)((3 * g * 8192) >> 4);
              const uint64_t kg = k_desc + (uint64_t)((slot * kKSlot) >> 4);
#pragma unroll
              for (int c = 0; c < 3; c++)
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                  mma_bf16_pair(tmem + kTmemS + sb * 64, qg + (uint64_t)((c * 8192 + kk * 32) >> 4),
                                kg + (uint64_t)((c * 8192 + kk * 32) >> 4), idesc_qk,
                                (g | c | kk) != 0 ? 1u : 0u);
              if (g + 1 < kKPerTile) {  // the last box is released by s_full
                tc_commit_pair(&sh->kempty[slot], 3);
                last_bar = &sh->kempty[slot];
                last_phase = u & 1;
              }
            }
            if (ok) {
              tc_commit_pair(&sh->s_full[sb], 3);
              last_bar = &sh->s_full[sb];
              last_phase = (gt >> 1) & 1;
            }
          }
          // both CTAs' Q may be reloaded once the unit's QK MMAs have completed
          if (ok) tc_commit_pair(&sh->q_empty, 3);
          nu++;
        }
      } else {
        const uint32_t idesc_pv = make_idesc(128, 256, kFmtBF16, kFmtBF16, false, true);
        const uint64_t p_desc = make_sdesc(p_addr, 16, 1024), v_desc = make_sdesc(v_addr, 8192, 1024);
        int nv = 0, gt = 0, nu = 0;  // V pages consumed, tiles, units
        for (UnitCursor c = cursor_begin(p, balanced, pair, npairs); c.pos < c.end && ok;
             cursor_next(p, balanced, c, npairs)) {
          const DecodeUnit U = cursor_unit(p, balanced, c, pair, npairs, rank);
          if (U.T <= 0) continue;
          // the first PV of a unit overwrites O: the previous epilogue has read it
          if (nu > 0 && !(ok = mbar_wait<true>(&sh->o_free, (nu - 1) & 1, abort))) break;
          for (int it = 0; it < U.T && ok; it++, gt++) {
            if (!(ok = mbar_wait<true>(&sh->p_full, gt & 1, abort))) break;
            tc_fence_after();
            for (int pg = 0; pg < kVPerTile; pg++, nv++) {
              const int slot = pg, u = gt;  // the ring holds one tile: page pg in slot pg
              if (!(ok = mbar_wait(&sh->vfull[slot], u & 1, abort))) break;
              // PV MMA j takes chunks 2j, 2j+1 of each CTA's slot: its output
              // columns are dims 256r + 128j + [0, 128) of CTA r's half
#pragma unroll
              for (int j = 0; j < 2; j++)
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                  // 16 tokens of page pg: P chunk pg, V slot rows 16kk..16kk+15
                  const uint64_t ad = p_desc + (uint64_t)((pg * 8192 + kk * 32) >> 4);
                  const uint64_t bd =
                      v_desc + (uint64_t)((slot * kVSlot + j * 16384 + kk * 2048) >> 4);
                  mma_bf16_pair(tmem + kTmemO + j * 128, ad, bd, idesc_pv,
                                (it > 0 || pg > 0 || kk > 0) ? 1u : 0u);
                }
              if (pg + 1 < kVPerTile) {  // the last page is released by p_free
                tc_commit_pair(&sh->vempty[slot], 3);
                last_bar = &sh->vempty[slot];
                last_phase = u & 1;
              }
            }
            if (ok) {
              tc_commit_pair(&sh->p_free, 3);
              last_bar = &sh->p_free;
              last_phase = gt & 1;
            }
          }
          if (ok) tc_commit_pair(&sh->o_full, 3);
          nu++;
        }
      }
      if (*abort && last_bar != nullptr) {
        // the MMAs issued so far finish before TMEM and the slots go away
        volatile int never = 0;
        mbar_wait<true>(last_bar, last_phase, &never);
      }
    }
  } else {
    // ------------------------------------------------ softmax / correction / epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane
    const int hl = row & 63, half = row >> 6;
    const int et = threadIdx.x - 64;      // 0..127 over warps 2-5
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    const uint32_t s_free_l[2] = {mapa_shared(smem_u32(&sh->s_free[0]), 0),
                                  mapa_shared(smem_u32(&sh->s_free[1]), 0)};
    const uint32_t p_full_l = mapa_shared(smem_u32(&sh->p_full), 0);
    const uint32_t o_free_l = mapa_shared(smem_u32(&sh->o_free), 0);
    // the last piece of a row (balanced schedule) marks the row's slots after
    // its own empty: weight zero in the combine
    auto mark_empty = [&](const DecodeUnit& U) {
      for (int slot = U.empty_from; slot < p.splits; slot++)
        for (int i = et; i < p.cta_heads; i += 128) {
          int blk;
          const int64_t prow = part_row_at(U.b, slot, U.head0 + i, blk);
          p.blk_ml[blk][prow * 2] = -INFINITY;
          p.blk_ml[blk][prow * 2 + 1] = 0.f;
        }
    };
    int gt = 0, nu = 0;  // tiles, units with tiles
    bool ok = true;
    for (UnitCursor c = cursor_begin(p, balanced, pair, npairs); c.pos < c.end && ok;
         cursor_next(p, balanced, c, npairs)) {
      const DecodeUnit U = cursor_unit(p, balanced, c, pair, npairs, rank);
      if (U.T <= 0) {
        if (p.direct) {  // no visible token: the output rows are zero
          for (int i = et; i < p.cta_heads * 64; i += 128)
            reinterpret_cast<uint4*>(out_row(U, U.head0 + (i >> 6)))[i & 63] =
                make_uint4(0u, 0u, 0u, 0u);
        } else {  // an empty partial: weight zero in the combine
          for (int i = et; i < p.cta_heads; i += 128) {
            int blk;
            const int64_t prow = part_row(U, U.head0 + i, blk);
            p.blk_ml[blk][prow * 2] = -INFINITY;
            p.blk_ml[blk][prow * 2 + 1] = 0.f;
          }
          mark_empty(U);
        }
        continue;
      }
      const int seqlen = U.seqlen, head0 = U.head0;
      float m_run = -INFINITY, l_run = 0.f;
      for (int it = 0; it < U.T && ok; it++, gt++) {
        const int sb = gt & 1;
        const uint32_t s_addr = tmem + lane_base + kTmemS + sb * 64;
        const int tok0 = (U.t_begin + it) * kTile + half * 64;
        const int nvalid = seqlen - tok0;  // tokens of this half that exist (may be <= 0 or > 64)
        if (!(ok = warp_wait(&sh->s_full[sb], (gt >> 1) & 1, abort))) break;
        tc_fence_after();
        // this thread's 64 scores into registers; the S buffer is then free
        float v[64];
#pragma unroll
        for (int c = 0; c < 2; c++)
          tmem_ld32(s_addr + c * 32, *reinterpret_cast<float(*)[32]>(v + 32 * c));
#pragma unroll
        for (int c = 0; c < 2; c++) tmem_ld_wait_regs(v + 32 * c);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(s_free_l[sb]);
        const bool full = nvalid >= 64;
        // pass 1: tile max
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int i = 0; i < 64; i++) mx = fmaxf(mx, v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 64; i++)
            if (i < nvalid) mx = fmaxf(mx, v[i]);
        }
        mx = (mx == -INFINITY) ? -INFINITY : mx * sl2;
        sh->xmax[sb][row] = mx;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->xbar[sb]);
        if (!(ok = warp_wait(&sh->xbar[sb], (gt >> 1) & 1, abort))) break;
        const float tmax = fmaxf(mx, sh->xmax[sb][row ^ 64]);
        float alpha = 1.f;
        bool resc = false;
        if (m_run == -INFINITY) {
          m_run = tmax;  // first tile: PV starts a fresh accumulator
        } else if (tmax > m_run + kRescale) {
          alpha = exp2f(m_run - tmax);
          m_run = tmax;
          resc = true;
        }
        // pass 2 into registers: P = 2^(s*scale*log2e - m) as bf16 pairs; the
        // row sum is over the unrounded values
        const uint64_t sc2 = f2_pack(sl2, sl2), nm2 = f2_pack(-m_run, -m_run);
        uint64_t sum2 = f2_pack(0.f, 0.f);
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
          const int e = 2 * i;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(v[e], v[e + 1]), sc2, nm2), x0, x1);
          float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
          if (!full) {
            p0 = (e < nvalid) ? p0 : 0.f;
            p1 = (e + 1 < nvalid) ? p1 : 0.f;
          }
          sum2 = f2_add(sum2, f2_pack(p0, p1));
          pk[i] = pack_bf16(p0, p1);
        }
        float ps0, ps1;
        f2_unpack(sum2, ps0, ps1);
        const float ps = ps0 + ps1;
        // P(t) reuses the buffer of P(t-1), and O holds tiles < t, once PV(t-1) is done
        if (gt >= 1 && !(ok = warp_wait(&sh->p_free, (gt - 1) & 1, abort))) break;
        // 64 tokens = one 128-byte row (chunk `half`, the page of CTA `half`)
        // of eight sixteen-byte units, swizzled
        uint8_t* pbase = sP + half * 8192 + hl * 128;
#pragma unroll
        for (int u = 0; u < 8; u++)
          *reinterpret_cast<uint4*>(pbase + ((u ^ (hl & 7)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        l_run = l_run * alpha + ps;
        if (__any_sync(0xffffffffu, resc)) {
          // rescale this warp's rows of O (PV(t-1) is complete): 256 columns
          // in two rounds of four loads in flight
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < 8; c0 += 4) {
            float o[4][32];
            const uint32_t ta = tmem + lane_base + kTmemO + c0 * 32;
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld32(ta + c * 32, o[c]);
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld_wait_regs(o[c]);
#pragma unroll
            for (int c = 0; c < 4; c++) {
#pragma unroll
              for (int i = 0; i < 32; i++) o[c][i] *= alpha;
              tmem_st32(ta + c * 32, o[c]);
            }
          }
          tmem_st_wait();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(p_full_l);
      }
      if (ok) ok = warp_wait(&sh->o_full, nu & 1, abort);
      sh->xsum[row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->lbar);
      if (ok) ok = warp_wait(&sh->lbar, nu & 1, abort);
      if (ok && p.direct) {
        // one split: sink and normalisation as attn_combine does for one part,
        // O / (l + 2^(sink*log2e - m)), rounded to bf16
        tc_fence_after();
        const float l_tot = l_run + sh->xsum[row ^ 64];
        float den;
        const float sk = (p.sink && hl < p.cta_heads) ? p.sink[head0 + hl] * kLog2e : -INFINITY;
        if (m_run != -INFINITY)
          den = l_tot + exp2f(sk - m_run);
        else
          den = l_tot + ((p.sink && hl < p.cta_heads && isfinite(p.sink[head0 + hl])) ? 1.f : 0.f);
        const float inv = 1.f / fmaxf(den, 1.17549435e-38f);
        __nv_bfloat16* po = out_row(U, head0 + hl) + 256 * half;
#pragma unroll 1
        for (int c = 0; c < 8; c++) {
          float v[32];
          tmem_ld32(tmem + lane_base + kTmemO + c * 32, v);
          tmem_ld_wait_regs(v);
          uint4* dst = reinterpret_cast<uint4*>(po + (c >> 2) * 128 + (c & 3) * 32);
          if (hl < p.cta_heads) {
#pragma unroll
            for (int i = 0; i < 4; i++)
              dst[i] = make_uint4(pack_bf16(v[8 * i] * inv, v[8 * i + 1] * inv),
                                  pack_bf16(v[8 * i + 2] * inv, v[8 * i + 3] * inv),
                                  pack_bf16(v[8 * i + 4] * inv, v[8 * i + 5] * inv),
                                  pack_bf16(v[8 * i + 6] * inv, v[8 * i + 7] * inv));
          }
        }
      } else if (ok) {
        tc_fence_after();
        const float l_tot = l_run + sh->xsum[row ^ 64];
        int blk = 0;
        const int64_t prow = hl < p.cta_heads ? part_row(U, head0 + hl, blk) : 0;
        const int64_t po = prow * 512 + 256 * half;  // element offset of this thread's half row
        const float inv_l = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll 1
        for (int c = 0; c < 8; c++) {
          float v[32];
          tmem_ld32(tmem + lane_base + kTmemO + c * 32, v);
          tmem_ld_wait_regs(v);
          const int64_t e = po + (c >> 2) * 128 + (c & 3) * 32;
          if (hl < p.cta_heads) {
            if (p.part_f16) {  // O / l in fp16: half the bytes, 2^-11 relative error
              uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.blk_o[blk]) + e);
#pragma unroll
              for (int i = 0; i < 4; i++)
                dst[i] = make_uint4(pack_f16(v[8 * i] * inv_l, v[8 * i + 1] * inv_l),
                                    pack_f16(v[8 * i + 2] * inv_l, v[8 * i + 3] * inv_l),
                                    pack_f16(v[8 * i + 4] * inv_l, v[8 * i + 5] * inv_l),
                                    pack_f16(v[8 * i + 6] * inv_l, v[8 * i + 7] * inv_l));
            } else {
              float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.blk_o[blk]) + e);
#pragma unroll
              for (int i = 0; i < 8; i++)
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          }
        }
        if (half == 0 && hl < p.cta_heads) {
          p.blk_ml[blk][prow * 2] = m_run;
          p.blk_ml[blk][prow * 2 + 1] = l_tot;
        }
        mark_empty(U);
      }
      // O is read: the next unit's first PV may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(o_free_l);
      nu++;
    }
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<2>(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort) raise_dev_error(p.err, QCAU_DEVERR_TIMEOUT);
  if (threadIdx.x == 0) signal_done(p);  // after the cluster barrier: both CTAs' stores
}

bool is_sm100_device() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

// CTA pairs of the kernel that can be resident at once on the current device
// (one CTA per SM, clusters of two), or 0 when the query fails.  Queried once
// per device, after the kernel's shared memory limit is set.
int resident_pairs() {
  static std::mutex mu;
  static int cached[64];
  static bool init = false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!init) {
    for (int& c : cached) c = -1;
    init = true;
  }
  if (cached[dev] < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, decode_attn_sm100_kernel, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace

bool decode_attn_sm100_supported(const AttnArgs& a) {
  // head blocks of q: the whole h, or divisors of 64 (8, 16, 32) and
  // multiples of 64 that divide h (the 1024-byte swizzle atom is 8 rows)
  const int64_t qhb = a.q_hblock > 0 ? a.q_hblock : a.h;
  const bool qblocks = qhb == a.h || (a.h % qhb == 0 && (qhb % 64 == 0 || (64 % qhb == 0 && qhb >= 8)));
  const bool parts = (a.o_hblock <= 0 || a.h % a.o_hblock == 0) &&
                     (a.part_hblock <= 0 || a.h % a.part_hblock == 0) &&
                     a.h / (a.part_hblock > 0 ? a.part_hblock : a.h) <= kMaxBlocks &&
                     (!a.peer || a.done_counter != nullptr);
  const bool ranges = a.splits_total <= 0 ||
                      (a.split_base >= 0 && a.split_base + a.splits <= a.splits_total);
  return qblocks && parts && ranges && a.block_table != nullptr && a.seqlens != nullptr &&
         a.s >= 1 && a.d_qk == 576 &&
         a.d_v == 512 && a.d_kv == 576 && a.page_size == 64 &&
         (a.h % 128 == 0 || a.h == 64 || a.h == 32 || a.h == 16) &&
         a.q_row_stride == 576 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.kv) & 15) == 0 && a.num_pages < (1LL << 31) &&
         a.max_pages < (1LL << 30) && is_sm100_device();
}

cudaError_t launch_decode_attn_sm100(const AttnArgs& a, cudaStream_t st) {
  if (!decode_attn_sm100_supported(a)) return cudaErrorNotSupported;
  // the balanced schedule: one query token per row, no fixed split range
  if (a.stream && (a.s != 1 || a.splits_total > 0 || a.peer || a.stream_nt < 1 ||
                   a.stream_usplits > a.splits ||
                   a.stream_pairs < 1 || (a.splits > 1 && a.part_o == nullptr)))
    return cudaErrorInvalidValue;
  if (a.b == 0) return cudaSuccess;
  // K and V are read through a 4-D view of the cache [pages][64 tokens][9
  // chunks][64 values], so that one box carries several chunks of a page: the
  // TMA engine's cost is per box, and 8 KB boxes cap a CTA at ~32 GB/s
  CUtensorMap tq, tk;
  // Q as [blocks][rows][q_hblock][576]: one block of h heads, or the ranks'
  // all-gathered head blocks (context-parallel decode)
  const int64_t rows = a.b * a.s;
  const int64_t qhb = a.q_hblock > 0 ? a.q_hblock : a.h;
  const int q_box = qhb < 64 ? (int)qhb : 64;
  {
    const uint64_t dims[4] = {576, (uint64_t)qhb, (uint64_t)rows, (uint64_t)(a.h / qhb)};
    const uint64_t strides[3] = {1152, (uint64_t)qhb * 1152, (uint64_t)(rows * qhb) * 1152};
    const uint32_t box[4] = {64, (uint32_t)q_box, 1, 1};
    if (!make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a.q, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  {
    // K: the same 4-D view, 3 chunks (24 KB) of one page per box
    const uint64_t dims[4] = {64, 64, 9, (uint64_t)a.num_pages};
    const uint64_t strides[3] = {1152, 128, 64 * 1152};
    const uint32_t box[4] = {64, 64, 3, 1};
    if (!make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a.kv, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  // V: the same 4-D view, 4 chunks (32 KB) of one page per box
  CUtensorMap tv;
  {
    const uint64_t dims[4] = {64, 64, 9, (uint64_t)a.num_pages};
    const uint64_t strides[3] = {1152, 128, 64 * 1152};
    const uint32_t box[4] = {64, 64, 4, 1};
    if (!make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, a.kv, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  }
  DecodeParams p;
  p.table = a.block_table;
  p.seqlens = a.seqlens;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.sink = a.sink;
  p.qlen = (int)a.s;
  p.q_hblock = (int)qhb;
  p.q_box = q_box;
  p.split_base = a.splits_total > 0 ? a.split_base : 0;
  const int usplits = a.stream && a.stream_usplits > 0 ? a.stream_usplits : (int)a.splits;
  p.usplits = usplits;
  p.splits_total = a.splits_total > 0 ? a.splits_total : usplits;
  p.part_hblock = a.part_hblock > 0 ? (int)a.part_hblock : (int)a.h;
  p.nblk = (int)(a.h / p.part_hblock);
  for (int j = 0; j < kMaxBlocks; j++) {
    p.blk_o[j] = nullptr;
    p.blk_ml[j] = nullptr;
    p.flag[j] = nullptr;
  }
  const int64_t blk_rows = rows * a.splits * p.part_hblock;
  for (int j = 0; j < p.nblk; j++) {
    if (a.peer) {  // receive slots of the ranks owning each block
      p.blk_o[j] = a.peer_o[j];
      p.blk_ml[j] = a.peer_ml[j];
      p.flag[j] = a.peer_flag[j];
    } else if (a.part_o) {
      p.blk_o[j] = reinterpret_cast<uint8_t*>(a.part_o) + j * blk_rows * 512 * (a.part_f16 ? 2 : 4);
      p.blk_ml[j] = a.part_ml + j * blk_rows * 2;
    }
  }
  p.counter = a.peer ? a.done_counter : nullptr;
  p.part_f16 = a.part_f16;
  p.o_hblock = a.o_hblock > 0 ? (int)a.o_hblock : (int)a.h;
  p.rows = rows;
  p.epoch = a.epoch;
  // one split and no partial buffers: the epilogue normalises and writes o
  p.direct = (a.splits == 1 && a.part_o == nullptr && !a.peer) ? 1 : 0;
  p.err = device_error_word();
  p.max_pages = a.max_pages;
  p.num_pages = a.num_pages;
  p.h = (int)a.h;
  p.cta_heads = a.h >= 128 ? 64 : (int)(a.h / 2);
  p.hgroups = (int)(a.h / (2 * p.cta_heads));
  p.splits = a.splits;
  p.scale = a.scale;
  cudaError_t e = cudaFuncSetAttribute(decode_attn_sm100_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  const int64_t units = a.b * a.s * usplits * p.hgroups;
  p.units = units;
  // one pair per unit; when the units outnumber the pairs that fit at once,
  // one pair per slot, each looping over units (no pair waits for another).
  // The balanced schedule has its own pair count (its ranges depend on it).
  const int64_t slots = resident_pairs();
  int64_t pairs = (slots > 0 && units > slots) ? slots : units;
  p.stream = a.stream ? 1 : 0;
  p.nt = a.stream_nt;
  p.gtiles = a.stream ? rows * p.hgroups * a.stream_nt : 0;
  if (a.stream) pairs = a.stream_pairs;
  decode_attn_sm100_kernel<<<(unsigned)(2 * pairs), kThreads, kSmemBytes, st>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace qcau
