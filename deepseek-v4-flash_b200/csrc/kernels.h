// kernels.h -- internal launchers of the QCAU sm_100a kernels (host side).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qcau {

// Host-side TMA descriptor builders (driver entry point resolved once).
// dims/strides innermost first; strides in bytes for dims 1..rank-1.
bool make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
               CUtensorMapSwizzle swizzle);

// Device address of the error word of the current device: a file-scope
// __device__ int in capi.cu (no allocation), resolved once per device.
int* device_error_word();

cudaError_t launch_act_quant(const void* x, void* y, void* s, int64_t m, int64_t n, int block,
                             int round_scale, int scale_e8m0, int inplace, cudaStream_t st);

cudaError_t launch_dequant_fp8_weight(const void* w, const void* s, int scale_e8m0, void* out,
                                      int64_t rows, int64_t cols, cudaStream_t st);

// RoPE of the rope part of rows (x points at the first rope value of row 0),
// in place, optionally also stored to `copy` rows; one thread per pair.
cudaError_t launch_rope_pairs(void* x, int64_t x_stride, void* copy, int64_t copy_stride,
                              const float* freqs, const int32_t* positions, int64_t b, int64_t s,
                              int64_t h, int rope_dim, int64_t pos0, int inverse,
                              cudaStream_t st);

cudaError_t launch_head_norm_rope(void* q, const void* gamma, const float* freqs,
                                  const int32_t* positions, int64_t b, int64_t s, int64_t h,
                                  int d, int64_t row_stride, int rope_dim, int64_t pos0,
                                  float eps, int do_norm, int do_rope, int inverse,
                                  cudaStream_t st);

// C[m,n] = two-level FP8 block-scaled GEMM (tcgen05).  out_f32: fp32 C.
cudaError_t launch_fp8_gemm(const void* a, const void* a_s, const void* b, const void* b_s,
                            void* c, int64_t m, int64_t n, int64_t k, int a_e8m0, int b_e8m0,
                            int out_f32, cudaStream_t st);

// The latent KV row of new tokens: RMSNorm (fp32, weight), RoPE of the last
// rope_dim values, FP8 block-64 round trip of the first quant_dims values,
// then the bf16 row to out[r] and to cache row slots[r] (kv_build.cu).
struct KvBuildArgs {
  const void* in;      // [rows, d] bf16 (the wkv projection)
  void* out;           // [rows, d] bf16 or nullptr (may equal in)
  int64_t rows, d;     // d a multiple of 64, <= 1024
  const float* norm_weight;  // [norm_dim] fp32 or nullptr (ones)
  int norm_dim;        // 0: no norm
  float eps;
  const float* freqs;  // [npos, rope_dim/2, 2] fp32
  const int32_t* positions;  // [rows]
  int64_t npos;
  int rope_dim;        // 0: no RoPE
  int quant_dims;      // a multiple of 64; 0: no FP8 round trip
  int round_scale;     // UE8M0 (power-of-two) scales
  void* cache;         // [cache_rows, d] bf16 or nullptr
  const int32_t* slots;  // [rows]: destination cache row, -1 to skip
  int64_t cache_rows;
  // seq_rows > 0 replaces positions and slots by arithmetic: row r is new row
  // i = r % seq_rows of sequence r / seq_rows, at position pos_base + i *
  // pos_step and cache row (r / seq_rows) * slot_seq_stride + slot_base + i
  int64_t seq_rows, pos_base, pos_step, slot_seq_stride, slot_base;
};
cudaError_t launch_kv_build(const KvBuildArgs& args, cudaStream_t st);

// Batched bf16 GEMM on tcgen05 for the absorbed-MLA projections:
//   for each batch g:  C_g[m, n] = A_g[m, k] . B_g^T  with
//   A_g row r at a + g*a_bstride + r*a_rstride (K contiguous),
//   B_g given either K-major (row j = output column, K contiguous, b_kmajor=1)
//   or MN-major (row t = K index, N contiguous, b_kmajor=0),
//   C_g row r at c + g*c_bstride + r*c_rstride (bf16).  Strides in elements.
struct BmmArgs {
  const void* a;
  int64_t a_bstride, a_rstride;
  const void* b;
  int64_t b_bstride, b_rstride;
  int b_kmajor;
  void* c;
  int64_t c_bstride, c_rstride;
  int64_t batch, m, n, k;
  int64_t b_rows;  // rows of B that exist (0: n); TMA zero-fills the rest
  // Optional act_quant of C in 1 x 128 blocks (act_quant.cu's arithmetic on
  // the bf16 values of C): codes at q_codes with C's element strides, scales
  // [m][c_rstride / 128] (fp32, or UE8M0 bytes with q_scale_e8m0).  Needs
  // n == 128 and c_bstride, c_rstride multiples of 128.
  void* q_codes;
  void* q_scales;
  int q_round_scale, q_scale_e8m0;
  // Optional RoPE of a 64-value rope slice per (row r of batch entry g),
  // done by the epilogue threads while the MMAs run (rope_norm.cu's
  // rope_pairs arithmetic): the slice at rope_x + (r * batch + g) *
  // rope_x_stride is rotated by rope_freqs[rope_pos[r]] (32 complex fp32),
  // written back in place and to rope_copy + (r * batch + g) *
  // rope_copy_stride.  Strides in elements, multiples of 8.
  void* rope_x;
  void* rope_copy;
  int64_t rope_x_stride, rope_copy_stride;
  const float* rope_freqs;
  const int32_t* rope_pos;
};
cudaError_t launch_bf16_bmm(const BmmArgs& args, cudaStream_t st);

// Indexer pieces (indexer.cu): the score scaling of its 128-wide rows
// (Walsh-Hadamard, FP4 e2m1 block-32 round trip), the weighted ReLU head sum
// of the raw scores with the prefill mask, the top-k selection, and the
// window / compressed index lists.
cudaError_t launch_rotate_fp4(void* x, int64_t rows, int hadamard, int fp4, cudaStream_t st);

// The indexer's score rows score[r, u] = bf16(sum_h bf16(relu(bf16(q[r, h] .
// kv[r / s, u])) * w[r, h])), fp32 [b * s, t], fused on tcgen05 (head_dim
// 128, h <= 128).
cudaError_t launch_indexer_score_sm100(const void* q, const void* kv, const void* w, float* score,
                                       int64_t b, int64_t s, int64_t h, int64_t t,
                                       int64_t kv_rows, cudaStream_t st);
cudaError_t launch_topk(const float* score, int64_t rows, int64_t t_len, int k, int32_t* out,
                        int64_t offset, int64_t s_len, int mask_ratio, cudaStream_t st);
// KV compressor gated pooling (compress.cu): prefill rows of the complete
// groups plus the state left behind, or one decode token into the state and,
// at a group boundary, its pooled row.
cudaError_t launch_compress(const float* kv, const float* score, const float* ape, float* kv_state,
                            float* score_state, void* out, int64_t bsz, int64_t seqlen, int d,
                            int ratio, int overlap, int64_t start_pos, cudaStream_t st);
cudaError_t launch_index_lists(int32_t* out, int64_t bsz, int64_t seqlen, int64_t start_pos,
                               int window, int ratio, int64_t offset, int win_w, int comp_w,
                               const int32_t* sel, cudaStream_t st);

// Split-KV attention arguments (gather by index or dense paged).
struct AttnArgs {
  const void* q;         // [rows, h, d_qk] where rows = b*s queries
  int64_t q_row_stride;  // elements between consecutive (query, head) rows
  const void* kv;        // dense [b, n_kv, d_kv] or paged [pages, page, d_kv]
  const int32_t* idx;    // [b*s, topk] indices (gather mode) or nullptr
  const int32_t* block_table;  // [b, max_pages] (paged mode) or nullptr
  const int32_t* seqlens;      // [b] (paged mode) or nullptr
  const float* sink;     // [h] or nullptr
  void* o;               // [rows, h, d_v] bf16
  float* part_o;         // [rows, splits, h, d_v] fp32 partials (splits > 1)
  float* part_ml;        // [rows, splits, h, 2] (max in log2 units, sum) partials
  int64_t b, s, h, d_qk, d_v, d_kv, n_kv, topk;
  int64_t page_size, max_pages, num_pages;
  int64_t max_len;       // topk (gather) or max seqlen (paged)
  int splits;
  float scale;
  // inverse RoPE epilogue (V4 QCAU): freqs [npos, rope/2, 2], pos = pos0 + t
  const float* freqs;
  int inv_rope;
  int rope_dim;
  int64_t pos0;
  // FP8 latent cache (gather mode, 576-wide rows): kv_fp8 [b, n_kv, 512]
  // e4m3, kv_scale [b, n_kv] fp32 per row, kv_rope [b, n_kv, 64] bf16; a
  // row's value is bf16(e4m3 * scale) followed by its rope part.  kv is unused.
  const uint8_t* kv_fp8;
  const float* kv_scale;
  const void* kv_rope;
  // Context-parallel decode over ranks (tcgen05 pair kernel; 0 = off):
  //   q is [h / q_hblock][rows][q_hblock][d_qk] (the ranks' all-gathered
  //   head blocks) when q_hblock > 0;
  //   this launch runs splits [split_base, split_base + splits) of
  //   splits_total over each row's tiles when splits_total > 0;
  //   partials go to [h / part_hblock][rows][splits][part_hblock] (one
  //   block per destination rank) when part_hblock > 0.
  int64_t q_hblock;
  int split_base, splits_total;
  int64_t part_hblock;
  // combine: partials are [splits][rows][h] (1) instead of [rows][splits][h]
  int part_split_major;
  // o as [h / o_hblock][rows][o_hblock][d_v] (the head owners' blocks) when
  // o_hblock > 0 (pair kernel's direct epilogue and the combine)
  int64_t o_hblock;
  // the O partials (part_o / peer_o) are O / sum in fp16 instead of
  // unnormalised O in fp32 (pair kernel writes, combine reads); the (max,
  // sum) partials stay fp32
  int part_f16;
  // Partials of head block j written straight into the receive slot of the
  // rank that owns it (peer memory), when peer != 0: peer_o[j] / peer_ml[j]
  // are [rows][splits][part_hblock] x d_v / x 2; the last CTA of the grid to
  // finish stores `epoch` to peer_flag[j] (release, system scope) and resets
  // done_counter (a zeroed device word of this GPU).
  int peer;
  void* peer_o[16];
  float* peer_ml[16];
  uint32_t* peer_flag[16];
  unsigned int* done_counter;
  uint32_t epoch;
  // Balanced decode schedule of the pair kernel (one query token per
  // sequence), when stream != 0: the tiles of every (row, head group), row
  // after row at max_len, are cut into stream_pairs equal ranges, one per
  // CTA pair; the pieces of a row, in pair order, are its partial slots, and
  // splits is the most pieces any row has.
  int stream;
  int64_t stream_nt;     // tiles of 128 tokens per row at max_len
  int64_t stream_pairs;
  int stream_usplits;    // the equal splits of the fall-back (<= splits; 0: splits)
};

// Wait (bounded, ~1 s) until flags[i] >= epoch (wrapping compare) for i < n;
// a timeout raises QCAU_DEVERR_TIMEOUT.  One block.
cudaError_t launch_wait_flags(const uint32_t* flags, int n, uint32_t epoch, cudaStream_t st);

// tcgen05 split-KV attention over gathered rows (attn_gather_sm100.cu): the
// top-k rows of each query (bf16, or FP8 codes + row scale + bf16 rope), or a
// paged cache in token order.  One split writes bf16 output (with the sink
// and the optional inverse RoPE); several write fp32 partials (part_o /
// part_ml, [rows][splits][h]) for attn_combine.
cudaError_t launch_attn_gather_sm100(const AttnArgs& args, cudaStream_t st);
bool attn_gather_sm100_supported(const AttnArgs& args);
// Heads per CTA of the gather kernel: 16, 32 or 64 (the MMAs' N).
int gather_heads_per_cta(int64_t h, int64_t d_qk);

// Merge split-KV partials into bf16 outputs (+ optional inverse RoPE)
// (attn_combine.cu).
cudaError_t launch_attn_combine(const AttnArgs& args, cudaStream_t st);

// tcgen05 two-CTA paged decode attention (h % 64 == 0, d_qk 576, d_v 512,
// page 64).  Writes partials for the combine kernel.
cudaError_t launch_decode_attn_sm100(const AttnArgs& args, cudaStream_t st);
bool decode_attn_sm100_supported(const AttnArgs& args);

}  // namespace qcau
