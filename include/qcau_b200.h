/*
 * qcau_b200.h -- C ABI of the B200 (sm_100a) QCAU path.
 *
 * The QCAU ("Query-Core Attention Unit") of DeepSeek-V4-Flash runs from the
 * q_lora activation c_q through the FP8 block-scaled query-up projection,
 * per-head RMSNorm and RoPE, MQA attention over a shared latent KV row with an
 * attention sink, and inverse RoPE.  This library implements it as
 * hand-written CUDA for sm_100a and also serves the absorbed-MLA decode layer
 * (query absorption into the latent space, dense paged decode attention,
 * v-up, FP8 output projection).
 *
 * Conventions
 *   - Every pointer is a device pointer unless the name says otherwise; all
 *     tensors are dense row-major (C-contiguous) with the shapes given.
 *   - bf16 tensors are passed as void*; FP8 tensors are float8_e4m3fn bytes;
 *     scale tensors are either fp32 or E8M0 bytes (value 2^(b-127)),
 *     selected by a qcau_scale_dtype argument.
 *   - Every call takes a cudaStream_t (passed as void*) and only enqueues
 *     work: no host synchronisation happens inside any entry point.
 *   - Return value: QCAU_OK (0) or a negative qcau_status.  On failure
 *     qcau_last_error() returns a message (thread-local).  Shape or dtype
 *     errors are reported before anything is enqueued.
 *   - Device-side anomalies (an index outside its range in a checked mode, a
 *     pipeline wait that timed out) set a device error word; read it with
 *     qcau_device_error() after the stream has been synchronised.
 *   - The library never allocates device memory on its own: callers pass a
 *     workspace where one is needed, sized by the matching *_workspace_size().
 *     The one allocating call is qcau_ipc_alloc, whose job it is (a buffer
 *     shared with peer processes through CUDA IPC).
 *
 * Reference file:line citations are relative to the reference project root
 * (dinhthituyetmai05/Deepseek-V4-Flash).
 */
#ifndef QCAU_B200_H
#define QCAU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    QCAU_OK = 0,
    QCAU_ERR_INVALID = -1,      /* shape / dtype / argument error  (ValueError) */
    QCAU_ERR_CUDA = -2,         /* CUDA runtime or driver error    (RuntimeError) */
    QCAU_ERR_UNSUPPORTED = -3,  /* valid but not implemented here  (NotImplementedError) */
    QCAU_ERR_WORKSPACE = -4,    /* workspace too small             (ValueError) */
    QCAU_ERR_DEVICE = -5        /* device error word was set        (RuntimeError) */
} qcau_status;

typedef enum { QCAU_SCALE_F32 = 0, QCAU_SCALE_E8M0 = 1 } qcau_scale_dtype;
typedef enum { QCAU_OUT_BF16 = 0, QCAU_OUT_F32 = 1 } qcau_out_dtype;

/* Device error word bits (qcau_device_error). */
#define QCAU_DEVERR_TIMEOUT 1   /* a bounded pipeline wait expired; the kernel returned early */
#define QCAU_DEVERR_INDEX 2     /* a block-table entry was outside [0, num_pages), or a
                                   decode sequence was longer than max_seqlen */

/* Library version (major*10000 + minor*100 + patch). */
int qcau_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* qcau_last_error(void);

/* Synchronise `stream`, read and clear the device error word of the current
 * device.  Returns the QCAU_DEVERR_* bits (0 = none) or a negative status. */
int qcau_device_error(void* stream);

/* ------------------------------------------------------------------------
 * act_quant -- replaces kernel.act_quant (Deepseek_origin/inference/
 * kernel.py:105-125, TileLang kernel :40-102; CPU restatement
 * QCAU/QCAU_inference/inference/kernel_fallback.py:48-64).
 *   x [m, n] bf16, n % block_size == 0.
 *   round_scale = 0: s = amax/448 (fp32);  1: s = 2^ceil(log2(amax/448))
 *   (scale_fmt="ue8m0", kernel.py:22-37).  amax is floored at 1e-4.
 *   inplace = 0: y [m, n] e4m3 codes, s [m, n/block] in scale_dtype.
 *   inplace = 1: x is overwritten with bf16(e4m3(x/s) * s); y and s unused
 *   (may be NULL).  Codes and scales are bit-exact with the reference.
 * ---------------------------------------------------------------------- */
int qcau_act_quant(const void* x, void* y, void* s, int64_t m, int64_t n,
                   int32_t block_size, int32_t round_scale, int32_t scale_dtype,
                   int32_t inplace, void* stream);

/* ------------------------------------------------------------------------
 * fp8_gemm -- replaces kernel.fp8_gemm (kernel.py:257-273, TileLang kernel
 * :203-254; C++ port qcau_c/src/qcau.cpp:30-90).
 *   c[m, n] = sum_kb (a[m, kb-block] . b[n, kb-block]) * a_s[m, kb] * b_s[n/128, kb]
 *   a [m, k] e4m3, a_s [m, k/128], b [n, k] e4m3, b_s [n/128, k/128];
 *   k % 128 == 0, n % 128 == 0; c [m, n] bf16 or fp32 (out_dtype).
 *   Each 128-wide K block is accumulated in fp32 on the tensor cores and then
 *   promoted with its two scales into a second fp32 accumulator, as the
 *   reference's two-level accumulation does.
 * ---------------------------------------------------------------------- */
int qcau_fp8_gemm(const void* a, const void* a_s, const void* b, const void* b_s,
                  void* c, int64_t m, int64_t n, int64_t k, int32_t scale_dtype,
                  int32_t out_dtype, void* stream);

/* ------------------------------------------------------------------------
 * head_norm_rope -- per-head RMSNorm (bf16 arithmetic, model.py:498,
 * QCAU/QCAU_inference/inference/QCAU.py:16-27, optional gamma [h, d]) followed
 * by RoPE of the last rope_dim values (model.py:231-243, QCAU.py:30-68), in
 * place on q [b, s, h, d] bf16.  freqs [npos, rope_dim/2, 2] fp32 (re, im);
 * row (b, t, .) uses freqs[pos0 + t].  do_norm = 0 skips the RMSNorm.
 * ---------------------------------------------------------------------- */
int qcau_head_norm_rope(void* q, const void* gamma, const float* freqs,
                        int64_t b, int64_t s, int64_t h, int64_t d,
                        int64_t row_stride, int64_t rope_dim, int64_t npos,
                        int64_t pos0, float eps, int32_t do_norm, void* stream);

/* RoPE alone, forward or inverse (conjugate), in place on rows of width d
 * (the rotated values are the last rope_dim of each row); model.py:231-243. */
int qcau_rope(void* x, const float* freqs, int64_t b, int64_t s, int64_t h,
              int64_t d, int64_t row_stride, int64_t rope_dim, int64_t npos,
              int64_t pos0, int32_t inverse, void* stream);

/* ------------------------------------------------------------------------
 * sparse_attn -- replaces kernel.sparse_attn (kernel.py:355-368, TileLang
 * kernel :276-352; QCAU.py:126-242; qcau_c/src/qcau.cpp:169-284).
 *   q [b, s, h, d_qk] bf16, kv [b, n_kv, d_kv] bf16 (d_kv >= d_qk),
 *   attn_sink [h] fp32 (NULL = no sink), topk_idxs [b, s, topk] int32,
 *   o [b, s, h, d_v] bf16 with V = kv[..., :d_v] (V4 model: d_v = d_qk = 512).
 *   Indices outside [0, n_kv) (the reference uses -1) are skipped.  P is
 *   rounded to bf16 before P.V as kernel.py:340 does; the sink enters the
 *   denominator once after the loop (kernel.py:345).  A query with no valid
 *   index returns zeros (QCAU.py:201-242 guard).
 *   inv_rope = 1 additionally applies the inverse RoPE of the last rope_dim
 *   values with freqs[pos0 + t] (QCAU.py:313-319) in the epilogue.
 * ---------------------------------------------------------------------- */
int qcau_sparse_attn(const void* q, const void* kv, const float* attn_sink,
                     const int32_t* topk_idxs, void* o, int64_t b, int64_t s,
                     int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                     int64_t n_kv, int64_t topk, float softmax_scale,
                     int32_t inv_rope, const float* freqs, int64_t rope_dim,
                     int64_t npos, int64_t pos0, void* stream);

/* ------------------------------------------------------------------------
 * qcau_forward -- the whole QCAU block, QCAU/QCAU_inference/inference/
 * QCAU.py:245-319 with w_uq given as the FP8 weight of wq_b
 * (ColumnParallelLinear, model.py:155-163 -> linear() :108-120):
 *   act_quant(c_q) -> fp8_gemm(wq_b) -> per-head RMSNorm -> RoPE ->
 *   sparse attention with sink -> inverse RoPE.
 *   c_q [b, s, dc] bf16; wq_b [h*d, dc] e4m3; wq_b_scale [h*d/128, dc/128];
 *   act_round_scale selects the activation scale format (1 = ue8m0, the
 *   model's scale_fmt); gamma [h, d] bf16 or NULL; kv [b, n_kv, d] bf16;
 *   topk_idxs [b, s, topk]; attn_sink [h]; freqs [npos, rope_dim/2, 2];
 *   o [b, s, h, d] bf16.  workspace >= qcau_forward_workspace_size(...).
 * ---------------------------------------------------------------------- */
size_t qcau_forward_workspace_size(int64_t b, int64_t s, int64_t h, int64_t d,
                                   int64_t dc);
int qcau_forward(const void* c_q, const void* wq_b, const void* wq_b_scale,
                 int32_t w_scale_dtype, int32_t act_round_scale, const void* gamma,
                 const void* kv, const int32_t* topk_idxs, const float* attn_sink,
                 const float* freqs, void* o, int64_t b, int64_t s, int64_t h,
                 int64_t d, int64_t dc, int64_t n_kv, int64_t topk,
                 int64_t rope_dim, int64_t npos, int64_t pos0, float norm_eps,
                 float softmax_scale, void* workspace, size_t workspace_bytes,
                 void* stream);

/* ------------------------------------------------------------------------
 * decode_attn_paged -- dense decode attention of one query token per
 * sequence over a paged latent cache (the decode branch of
 * Attention.forward, model.py:529-533, with the window/compressed index list
 * replaced by "all cached tokens"; same numerics as sparse_attn).
 *   q [b, h, d_qk] bf16; cache [num_pages, page_size, d_kv] bf16;
 *   block_table [b, max_pages] int32; seqlens [b] int32 (tokens per
 *   sequence, <= max_seqlen <= max_pages*page_size); attn_sink [h] or NULL;
 *   o [b, h, d_v] bf16 (V = cache row[:d_v]).
 *   Split-KV: partial results go to the workspace and a combine kernel
 *   merges them (workspace >= qcau_decode_attn_workspace_size(...)).  The
 *   two-CTA kernel schedules every sequence at max_seqlen: a longer one is
 *   cut there and raises QCAU_DEVERR_INDEX.
 *   On sm_100a with h a multiple of 128 or h in {16, 32, 64}, d_qk == 576,
 *   d_v == 512, page_size == 64
 *   this runs the tcgen05 two-CTA kernel; other shapes run the general
 *   split-KV kernel.
 * ---------------------------------------------------------------------- */
size_t qcau_decode_attn_workspace_size(int64_t b, int64_t h, int64_t d_v,
                                       int64_t max_seqlen);
int qcau_decode_attn_paged(const void* q, const void* cache,
                           const int32_t* block_table, const int32_t* seqlens,
                           const float* attn_sink, void* o, int64_t b, int64_t h,
                           int64_t d_qk, int64_t d_v, int64_t d_kv,
                           int64_t page_size, int64_t max_pages, int64_t num_pages,
                           int64_t max_seqlen, float softmax_scale, void* workspace,
                           size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * decode_attn_paged_blocked -- decode_attn_paged with q and o in head blocks
 * (no reference counterpart): q [h / q_hblock, b, q_hblock, d_qk] and o
 * [h / o_hblock, b, o_hblock, d_v], the layouts in which head-sharded ranks
 * hand each other the query and output rows of the sequences one rank
 * attends (see the layer stages below).  Same workspace, kernels, split
 * counts and results as decode_attn_paged; needs the sm_100a pair kernel
 * (d_qk 576, d_v 512, page 64, h a multiple of 128, each head block a
 * multiple of 64 or one of 8, 16, 32) and returns QCAU_ERR_UNSUPPORTED
 * otherwise.
 * ---------------------------------------------------------------------- */
int qcau_decode_attn_paged_blocked(const void* q, int64_t q_hblock, const void* cache,
                                   const int32_t* block_table, const int32_t* seqlens,
                                   const float* attn_sink, void* o, int64_t o_hblock, int64_t b,
                                   int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                                   int64_t page_size, int64_t max_pages, int64_t num_pages,
                                   int64_t max_seqlen, float softmax_scale, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * sparse_attn_fp8 -- sparse_attn (kernel.py:355-368) over an FP8 latent
 * cache: top-k gather decode at long context with the latent part stored as
 * e4m3 codes and one fp32 scale per row, the rope part in bf16.  The
 * reference keeps its FP8 round trip in a bf16 cache (act_quant inplace,
 * model.py:505); this layout stores the codes themselves (644 bytes per row
 * instead of 1152) and dequantises each gathered row to
 * bf16(e4m3 * scale) before the same attention as sparse_attn (576-wide K,
 * V = the 512 latent values, bf16 P, sink once, index -1 skipped).
 *   q [b, s, h, 576] bf16; kv_latent [b, n_kv, 512] e4m3 (16-byte aligned);
 *   kv_scale [b, n_kv] fp32; kv_rope [b, n_kv, 64] bf16 (16-byte aligned);
 *   topk_idxs [b, s, topk] int32; o [b, s, h, 512] bf16;
 *   workspace >= qcau_sparse_attn_fp8_workspace_size(...) (split-KV partials).
 * ---------------------------------------------------------------------- */
size_t qcau_sparse_attn_fp8_workspace_size(int64_t b, int64_t s, int64_t h, int64_t topk);
int qcau_sparse_attn_fp8(const void* q, const void* kv_latent, const float* kv_scale,
                         const void* kv_rope, const float* attn_sink,
                         const int32_t* topk_idxs, void* o, int64_t b, int64_t s,
                         int64_t h, int64_t n_kv, int64_t topk, float softmax_scale,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * prefill_attn_paged -- causal attention of s new query tokens per sequence
 * over the paged latent cache that already holds them (prefill, chunked
 * prefill, multi-token decode): the prefill branch of Attention.forward
 * (model.py:484-543), whose causal window index lists
 * (get_window_topk_idxs, model.py:254-264) become "every cached token up to
 * the query's position"; same numerics as sparse_attn.
 *   q [b, s, h, d_qk] bf16; o [b, s, h, d_v] bf16; cache / block_table as
 *   decode_attn_paged; seqlens [b] = cached tokens of each sequence,
 *   including its s new ones (>= s).  Token t of sequence i attends to
 *   cache positions [0, seqlens[i] - s + t].
 *   workspace >= qcau_prefill_attn_workspace_size(...) (zero when the KV
 *   range is not split, e.g. at prefill sizes: the kernel then normalises and
 *   writes o itself).  Kernels as decode_attn_paged.
 * ---------------------------------------------------------------------- */
size_t qcau_prefill_attn_workspace_size(int64_t b, int64_t s, int64_t h, int64_t d_v,
                                        int64_t max_seqlen);
int qcau_prefill_attn_paged(const void* q, const void* cache,
                            const int32_t* block_table, const int32_t* seqlens,
                            const float* attn_sink, void* o, int64_t b, int64_t s,
                            int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                            int64_t page_size, int64_t max_pages, int64_t num_pages,
                            int64_t max_seqlen, float softmax_scale, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * decode_attn_paged_noalloc -- qcau_decode_attn_paged for callers that
 * cannot allocate device memory.  No counterpart in the reference: its
 * kernels allocate through PyTorch; this entry point exists only for the
 * no-cudaMalloc case.
 *   Same arguments, kernels, split counts and results as
 *   qcau_decode_attn_paged, but the split-KV partials live in a file-scope
 *   static device array of QCAU_DECODE_STATIC_SCRATCH_BYTES (32 MiB), which
 *   every device that loads this library holds until the process exits.
 *   Allocates nothing: no cudaMalloc/cudaFree and no allocating library call.
 *   Inputs whose partials need more than that (qcau_decode_attn_workspace_size
 *   > QCAU_DECODE_STATIC_SCRATCH_BYTES, e.g. batch 128 x 128 heads at 32K
 *   context) are rejected with QCAU_ERR_WORKSPACE before any device work.
 *   The scratch address is resolved once per device (cudaGetSymbolAddress
 *   with that device current) and kept until the process exits; make the
 *   first call on each device outside any stream capture.  A reset of the
 *   device's primary context (cudaDeviceReset) while the library is loaded
 *   is not supported: the kept address would be stale.  Nothing in the
 *   scratch must start at zero: every
 *   partial row the combine reads is written earlier in the same call.
 *   There is ONE scratch per device: calls whose executions overlap on the
 *   same device (two streams, or two host threads) race on it and give
 *   wrong results.  Calls ordered on one stream are safe.
 * ---------------------------------------------------------------------- */
#define QCAU_DECODE_STATIC_SCRATCH_BYTES ((size_t)32 << 20)
int qcau_decode_attn_paged_noalloc(const void* q, const void* cache,
                                   const int32_t* block_table, const int32_t* seqlens,
                                   const float* attn_sink, void* o, int64_t b, int64_t h,
                                   int64_t d_qk, int64_t d_v, int64_t d_kv,
                                   int64_t page_size, int64_t max_pages, int64_t num_pages,
                                   int64_t max_seqlen, float softmax_scale, void* stream);

/* ------------------------------------------------------------------------
 * gopu -- the V4 output side of the attention block after the QCAU output
 * o (Deepseek_origin/inference/model.py:536-542): the grouped low-rank
 * projection wo_a (einsum "bsgd,grd->bsgr", a bf16 weight) and the
 * row-parallel wo_b (RowParallelLinear :166-180 -> linear() :108-120:
 * act_quant of the activation, FP8 GEMM with 128x128 block scales).
 *   o [rows, groups, group_dim] bf16 (the heads of a group side by side:
 *   group_dim = heads / groups * head_dim); wo_a [groups, rank_dim,
 *   group_dim] bf16; wo_b [dim, groups*rank_dim] e4m3 + wo_b_scale
 *   [dim/128, groups*rank_dim/128] (scale_dtype); y [rows, dim] bf16 or
 *   fp32 (out_dtype).  act_round_scale selects UE8M0 activation scales (the
 *   model's scale_fmt).  A head shard passes its own groups and wo_b
 *   columns; the partial y of the ranks is summed by the caller (the
 *   reference all-reduces in fp32, model.py:174-177).
 *   Workspace: qcau_gopu_workspace_size(rows, groups, rank_dim).
 * ---------------------------------------------------------------------- */
size_t qcau_gopu_workspace_size(int64_t rows, int64_t groups, int64_t rank_dim);
int qcau_gopu(const void* o, const void* wo_a, const void* wo_b, const void* wo_b_scale,
              int32_t scale_dtype, int32_t act_round_scale, void* y, int32_t out_dtype,
              int64_t rows, int64_t groups, int64_t group_dim, int64_t rank_dim,
              int64_t dim, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * kv_build -- the latent KV row of new tokens, from the wkv projection to the
 * cache: Deepseek_origin/inference/model.py:502-506 (kv_norm, RoPE of the
 * last rope_dim values, act_quant(kv[..., :-rd], 64, scale_fmt, inplace))
 * and the cache writes :517-533 (window ring kv_cache[b, pos % win]), also
 * the Compressor's tail :362-376 on its pooled rows.
 *   kv_in [rows, d] bf16 (d a multiple of 64, <= 1024); kv_out [rows, d]
 *   bf16 or NULL, may equal kv_in;
 *   norm_weight [norm_dim] fp32 or NULL (ones); norm_dim 0 (no norm), or a
 *   multiple of 64 <= d: RMSNorm of values [0, norm_dim) in fp32
 *   (model.py:182-195);
 *   freqs [npos, rope_dim/2, 2] fp32, positions [rows] int32: RoPE of the
 *   last rope_dim values (rope_dim 0: none);
 *   quant_dims: a multiple of 64 <= d - rope_dim: FP8 e4m3 round trip of
 *   values [0, quant_dims) in 1x64 blocks, UE8M0 scales with round_scale
 *   (scale_fmt "ue8m0") else fp32 amax/448;
 *   cache [cache_rows, d] bf16 or NULL; cache_slots [rows] int32: the cache
 *   row of each input row, -1 to skip (a window ring: b * ring + pos % win;
 *   a paged cache: page * page_size + pos % page_size).
 * A position or slot out of range is skipped and raises QCAU_DEVERR_INDEX.
 * ---------------------------------------------------------------------- */
int qcau_kv_build(const void* kv_in, void* kv_out, int64_t rows, int64_t d,
                  const float* norm_weight, int64_t norm_dim, float eps,
                  const float* freqs, const int32_t* positions, int64_t npos,
                  int64_t rope_dim, int64_t quant_dims, int32_t round_scale,
                  void* cache, const int32_t* cache_slots, int64_t cache_rows,
                  void* stream);

/* ------------------------------------------------------------------------
 * compress -- the KV compressor's gated pooling, Compressor.forward
 * (QCAU/QCAU_inference/inference/model.py:415-457; Deepseek_origin/inference/
 * model.py:317-357) after its two fp32 projections:
 *   kv, score [bsz, seqlen, cw] fp32 = wkv(x.float()), wgate(x.float()),
 *   cw = 2d with overlap (the ratio-4 compressor), else d;
 *   ape [ratio, cw] fp32; kv_state, score_state [bsz, slots, cw] fp32 with
 *   slots = 2 * ratio (overlap) or ratio, the compressor's decode state.
 * Prefill (start_pos 0): out [bsz, seqlen / ratio, d] bf16 = per channel the
 *   softmax(score + ape)-weighted sum of each group's kv (with overlap the
 *   window is the previous group on channels [0, d) and this group on
 *   [d, 2d), model.py:406-413), rounded to bf16; the state (may be NULL) is
 *   left as the reference leaves it: the last complete group (overlap) and
 *   the remainder tokens, scores with ape added (model.py:422-429).
 * Decode (seqlen 1, start_pos > 0): the token goes into the state; when
 *   (start_pos + 1) % ratio == 0, out [bsz, d] bf16 is the pooled state (and
 *   with overlap the state shifts by one group); else out is not written.
 * The pooled rows then take the compressor's norm, RoPE and quantisation
 * through qcau_kv_build (model.py:459-476).
 * ---------------------------------------------------------------------- */
int qcau_compress(const float* kv, const float* score, const float* ape, float* kv_state,
                  float* score_state, void* out, int64_t bsz, int64_t seqlen, int64_t d,
                  int64_t ratio, int32_t overlap, int64_t start_pos, void* stream);

/* ------------------------------------------------------------------------
 * compressor_step -- one whole Compressor.forward after its projections
 * (QCAU/QCAU_inference/inference/model.py:415-476; Deepseek_origin/inference/
 * model.py:317-377): qcau_compress's pooling, then on the compressed rows the
 * kv_norm RMSNorm over all d values (fp32 norm_weight, NULL = ones), RoPE of
 * the last rope_dim values at each row's first position, and either the FP8
 * round trip of the values below the rope part (rotate 0, the attention's
 * compressor) or the Hadamard rotation and FP4 round trip of qcau_rotate_fp4
 * (rotate 1, the indexer's, d = 128); the rows are written to rows_out
 * [bsz, n, d] bf16 and, when cache is not NULL, to the caller's cache
 * [>= bsz, cache_seq_rows, d] bf16 at rows cache_offset + first + i of each
 * sequence (model.py:472-475; the attention's compressed rows follow its
 * window ring, cache_offset = window_size).  n = seqlen / ratio and first =
 * 0 at a prefill (start_pos 0); at a decode step n = 1 when (start_pos + 1)
 * % ratio == 0, else 0 (only the state is updated), and first = start_pos /
 * ratio.  Row i sits at position (first + i) * ratio of freqs [npos,
 * rope_dim/2, 2] fp32.  Positions and cache rows are computed on the device,
 * so a decode step is two or three launches and no host-side tensors.
 * ---------------------------------------------------------------------- */
int qcau_compressor_step(const float* kv, const float* score, const float* ape, float* kv_state,
                         float* score_state, int64_t bsz, int64_t seqlen, int64_t d,
                         int64_t ratio, int32_t overlap, int64_t start_pos,
                         const float* norm_weight, float eps, const float* freqs, int64_t npos,
                         int64_t rope_dim, int32_t rotate, int32_t round_scale, void* cache,
                         int64_t cache_seq_rows, int64_t cache_offset, void* rows_out,
                         void* stream);

/* ------------------------------------------------------------------------
 * Index-list producers: what the sparse attention's topk_idxs come from.
 *
 * qcau_rotate_fp4 -- in place on rows of 128 bf16 values: the Walsh-Hadamard
 *   rotation rotate_activation (QCAU/QCAU_inference/inference/model.py:302-
 *   323: Sylvester order, fp32 butterflies, times 128^-1/2, back to bf16;
 *   the reference's own restatement of the third-party fast_hadamard_
 *   transform) when `hadamard`, then, when `fp4`, fp4_act_quant(x, 32,
 *   inplace=True) (Deepseek_origin/inference/kernel.py:128-200: per 1x32
 *   block s = 2^ceil(log2(max(amax, 6*2^-126) * (1/6))), x/s clamped to
 *   +-6 and rounded to FP4 e2m1, times s, to bf16).  The Indexer applies both
 *   to its queries (model.py:512-514) and its Compressor to the pooled key
 *   rows (model.py:466-468).  d must be 128.
 *
 * qcau_indexer_topk -- Indexer.forward after the projections
 *   (model.py:518-533): with q [b, s, h, d] bf16 (rotated + FP4), kv the
 *   indexer's compressed cache [b, kv_rows, d] bf16 of which the first
 *   t = end_pos / ratio rows of each sequence are read,
 *   weights [b, s, h] bf16 (weights_proj(x) * softmax_scale * h^-1/2),
 *     score[b, s, u] = bf16(sum_h bf16(relu(bf16(q[b,s,h] . kv[b,u])) * w[b,s,h]))
 *   masked to -inf at prefill (start_pos == 0) where u >= (s + 1) / ratio,
 *   then topk_idxs [b, s, k] int32 = the k largest per row (score
 *   descending, equal scores by index ascending) + offset; entries past a
 *   row's finite scores are -1, as the reference's mask makes them.  k is
 *   min(index_topk, t) in the reference (<= 2048 here); d must be 128 (the
 *   model's index_head_dim) and h <= 128.  The score rows are computed in
 *   one pass over the keys: the einsum's [b, s, h, t] output stays on chip.
 *   The workspace holds the score rows:
 *   qcau_indexer_topk_workspace_size(b, s, h, t) bytes.
 *   Its two halves, for head-sharded ranks that all-reduce the score rows
 *   between them (model.py:520-521):
 *   qcau_indexer_scores -- score [b, s, t] fp32 (bf16 values), unmasked;
 *     qcau_indexer_scores_workspace_size(b, s, h, t) is 0 (no workspace).
 *   qcau_topk -- topk_idxs [rows, k] of score [rows, t]: the k largest of a
 *     row, score descending then index ascending, + offset, -1 past the
 *     row's candidates; -inf is never taken, and with mask_ratio > 0 (a
 *     prefill: the indexer's ratio) neither are positions >= (row % seqlen
 *     + 1) / mask_ratio.  A drop-in for score.topk(k, dim=-1)[1] whenever
 *     the row's k-th score has no equal outside the selection.
 *
 * qcau_index_lists -- the [bsz, seqlen, W] int32 index list the attention
 *   reads: get_window_topk_idxs(window, bsz, seqlen, start_pos)
 *   (model.py:326-357) followed by either `selected` [bsz, seqlen,
 *   selected_width] (the indexer's list, offset included) or, when
 *   `selected` is NULL and ratio > 0, get_compress_topk_idxs(ratio, bsz,
 *   seqlen, start_pos, offset) (model.py:359-376), as Attention.forward
 *   concatenates them (model.py:614-624).  W = qcau_index_lists_width(...).
 *   Decode steps (start_pos > 0) have seqlen 1.
 * ---------------------------------------------------------------------- */
int qcau_rotate_fp4(void* x, int64_t rows, int64_t d, int32_t hadamard, int32_t fp4,
                    void* stream);
size_t qcau_indexer_topk_workspace_size(int64_t b, int64_t s, int64_t h, int64_t t);
size_t qcau_indexer_scores_workspace_size(int64_t b, int64_t s, int64_t h, int64_t t);
/* qcau_indexer_raw_scores -- the einsum alone, raw [b, s * h, round_up(t,
 *   128)] bf16 = q[b, s, h, :] . kv[b, u, :] (model.py:518; columns past t
 *   are zero): the intermediate the fused score pass keeps on chip, for
 *   inspection; d a multiple of 64, any h. */
int qcau_indexer_raw_scores(const void* q, const void* kv, void* raw, int64_t b, int64_t s,
                            int64_t h, int64_t d, int64_t t, int64_t kv_rows, void* stream);
int qcau_indexer_scores(const void* q, const void* kv, const void* weights, float* score,
                        int64_t b, int64_t s, int64_t h, int64_t d, int64_t t, int64_t kv_rows,
                        void* workspace, size_t workspace_bytes, void* stream);
int qcau_topk(const float* score, int32_t* topk_idxs, int64_t rows, int64_t t, int64_t k,
              int64_t seqlen, int64_t mask_ratio, int64_t offset, void* stream);
int qcau_indexer_topk(const void* q, const void* kv, const void* weights, int32_t* topk_idxs,
                      int64_t b, int64_t s, int64_t h, int64_t d, int64_t t, int64_t kv_rows,
                      int64_t k, int64_t start_pos, int64_t ratio, int64_t offset,
                      void* workspace, size_t workspace_bytes, void* stream);
int64_t qcau_index_lists_width(int64_t seqlen, int64_t start_pos, int64_t window,
                               int64_t ratio, int64_t selected_width);
int qcau_index_lists(int32_t* topk_idxs, int64_t bsz, int64_t seqlen, int64_t start_pos,
                     int64_t window, int64_t ratio, int64_t offset, const int32_t* selected,
                     int64_t selected_width, void* stream);

/* ------------------------------------------------------------------------
 * Absorbed-MLA decode layer (BASELINE decode configs; the reference's V4
 * attention has no wkv_b, so these extend its surface).  Weights:
 *   wq_b   [h*(d_nope+d_rope), dc] e4m3 + scale [.. /128, dc/128]
 *   wkv_b  [h*(d_nope+d_v), kv_lora] bf16 (dequantised once from FP8 by
 *          qcau_dequant_fp8_weight)
 *   wo     [dim, h*d_v] e4m3 + scale [dim/128, h*d_v/128]   (row-parallel)
 * Per step:
 *   act_quant(q_lora) -> fp8_gemm(wq_b) -> RoPE(q_rope at positions[b]) ->
 *   absorb q_nope . W_UK -> decode_attn_paged -> v-up o_lat . W_UV ->
 *   act_quant -> fp8_gemm(wo) -> y [b, dim] (bf16 or fp32, to be summed
 *   over head shards by the caller's all-reduce, as RowParallelLinear does,
 *   model.py:166-180).
 * ---------------------------------------------------------------------- */
typedef struct {
    int64_t batch;       /* sequences, one query token each            */
    int64_t n_heads;     /* local heads on this rank                   */
    int64_t dc;          /* q_lora_rank                                */
    int64_t d_nope;      /* 128                                        */
    int64_t d_rope;      /* 64                                         */
    int64_t kv_lora;     /* 512                                        */
    int64_t d_v;         /* 128                                        */
    int64_t dim;         /* model width of the o-projection output     */
    int64_t page_size;   /* 64                                         */
    int64_t max_pages;   /* block_table row length                     */
    int64_t num_pages;   /* physical pages in the cache                */
    int64_t max_seqlen;  /* upper bound of seqlens[]                   */
    int64_t npos;        /* rows of freqs                              */
    float softmax_scale;
    int32_t w_scale_dtype;   /* scale format of wq_b / wo scales        */
    int32_t act_round_scale; /* 1: ue8m0 activation scales              */
    int32_t out_dtype;       /* y dtype                                 */
} qcau_mla_dims;

/* FP8 weight with 128x128 block scales -> bf16 (one-time weight preparation). */
int qcau_dequant_fp8_weight(const void* w, const void* w_scale, int32_t scale_dtype,
                            void* out_bf16, int64_t rows, int64_t cols, void* stream);

size_t qcau_mla_decode_workspace_size(const qcau_mla_dims* dims);
int qcau_mla_decode(const qcau_mla_dims* dims, const void* q_lora,
                    const void* wq_b, const void* wq_b_scale, const void* wkv_b_bf16,
                    const void* wo, const void* wo_scale, const void* cache,
                    const int32_t* block_table, const int32_t* seqlens,
                    const int32_t* positions, const float* freqs, void* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * The layer in stages, for head-sharded ranks that split the attention by
 * context instead of each streaming the whole shared cache (no reference
 * counterpart: its ranks run Attention.forward on their heads, model.py:
 * 484-543, and meet only in RowParallelLinear's all-reduce, model.py:166-180).
 * With N ranks, rank r owning heads [r*h/N, (r+1)*h/N):
 *   mla_decode_q        q_abs [b, h/N, kv_lora+d_rope] of its heads
 *   (caller)            all-gather -> q_all [N, b, h/N, 576]
 *   decode_attn_paged_cp   all h heads over tiles [ntiles*r/N, ntiles*(r+1)/N)
 *                       of every sequence (ntiles = ceil(seqlen/128)) ->
 *                       partials [N, b, h/N, 512] (unnormalised O in
 *                       fp32, or with part_f16 = 1 O / sum in fp16: half
 *                       the bytes to exchange) and [N, b, h/N, 2] fp32
 *                       (max in log2 units, sum), block j holding the heads
 *                       of rank j
 *   (caller)            all-to-all of the blocks -> [N, b, h/N, ...] by source
 *   attn_combine_ranks  o_lat [b, h/N, 512] bf16 (sink optional)
 *   mla_decode_out      y [b, dim] (row-parallel partial)
 *   (caller)            all-reduce of y
 * Every stage takes qcau_mla_dims with n_heads = h/N (the rank's heads) and
 * the workspace of qcau_mla_decode_workspace_size.  The partials hold
 * (O, max in log2 units, sum) as the split-KV path does;
 * decode_attn_paged_cp needs the sm_100a pair kernel (d_qk 576, d_v 512,
 * page 64, h a multiple of 128, h/N a multiple of 64 or one of 8, 16, 32)
 * and returns QCAU_ERR_UNSUPPORTED otherwise.
 * ---------------------------------------------------------------------- */
int qcau_mla_decode_q(const qcau_mla_dims* dims, const void* q_lora, const void* wq_b,
                      const void* wq_b_scale, const void* wkv_b_bf16,
                      const int32_t* positions, const float* freqs, void* q_abs,
                      void* workspace, size_t workspace_bytes, void* stream);
int qcau_decode_attn_paged_cp(const void* q_all, const void* cache,
                              const int32_t* block_table, const int32_t* seqlens,
                              void* part_o, float* part_ml, int64_t b, int64_t h,
                              int64_t n_ranks, int64_t rank, int64_t d_qk, int64_t d_v,
                              int64_t d_kv, int64_t page_size, int64_t max_pages,
                              int64_t num_pages, int64_t max_seqlen, float softmax_scale,
                              int32_t part_f16, void* stream);
int qcau_attn_combine_ranks(const void* part_o, const float* part_ml, const float* attn_sink,
                            void* o, int64_t b, int64_t h_local, int64_t n_ranks, int64_t d_v,
                            int32_t part_f16, void* stream);
int qcau_mla_decode_out(const qcau_mla_dims* dims, const void* o_lat, const void* wkv_b_bf16,
                        const void* wo, const void* wo_scale, void* y, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * The exchange of decode_attn_paged_cp fused into the attention kernel (no
 * reference counterpart).  Each rank owns a receive buffer in its own GPU
 * memory, exported through CUDA IPC (ipc_alloc, zero-filled; handles of
 * qcau_ipc_handle_size() bytes swapped between the processes by the
 * caller; ipc_open maps a peer's buffer, with peer access over NVLink).
 * decode_attn_paged_cp_p2p computes what decode_attn_paged_cp does, but
 * writes the partials of head block j (the heads of rank j) straight into
 * rank j's buffer: dst_o[j] -> [b, h/N, d_v] (fp32, or fp16 with part_f16)
 * and dst_ml[j] ->
 * [b, h/N, 2], this rank's slot of rank j's [N_src, b, h/N, ...] receive
 * area.  The last CTA to finish then stores `epoch` to dst_flag[j] (this
 * rank's flag word in rank j's buffer) with release semantics at system
 * scope; done_counter is a zeroed uint32 of this GPU that the kernel
 * resets.  wait_flags (one block, bounded at ~1 s, then
 * QCAU_DEVERR_TIMEOUT) waits until the n flags of this rank's buffer reach
 * `epoch` (wrapping compare); the receive area is then complete.
 * All ranks call with the same b (b == 0 writes and signals nothing).  A
 * receive area must not be rewritten before its owner has merged it: the
 * caller alternates two areas by step and orders steps (the layer's
 * all-reduce of y does).  Pointers in dst_* are device pointers; the arrays
 * themselves are host memory of n_ranks entries (n_ranks <= 16).
 * ---------------------------------------------------------------------- */
size_t qcau_ipc_handle_size(void);
int qcau_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
int qcau_ipc_open(const void* handle, void** ptr);
int qcau_ipc_close(void* ptr);
int qcau_ipc_free(void* ptr);
int qcau_decode_attn_paged_cp_p2p(const void* q_all, const void* cache,
                                  const int32_t* block_table, const int32_t* seqlens,
                                  void* const* dst_o, float* const* dst_ml,
                                  uint32_t* const* dst_flag, uint32_t epoch,
                                  uint32_t* done_counter, int64_t b, int64_t h, int64_t n_ranks,
                                  int64_t rank, int64_t d_qk, int64_t d_v, int64_t d_kv,
                                  int64_t page_size, int64_t max_pages, int64_t num_pages,
                                  int64_t max_seqlen, float softmax_scale, int32_t part_f16,
                                  void* stream);
int qcau_wait_flags(const uint32_t* flags, int64_t n, uint32_t epoch, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QCAU_B200_H */
