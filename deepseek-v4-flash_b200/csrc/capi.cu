// capi.cu -- the C ABI (include/qcau_b200.h): argument validation, error
// reporting, workspace layout and the orchestration of the multi-kernel
// entry points.  No entry point synchronises the host or allocates device
// memory; qcau_device_error() is the only call that synchronises.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include <cstring>

using namespace qcau;

// ---------------------------------------------------------------- errors

static thread_local std::string g_last_error;

static int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

static int fail_cuda(cudaError_t e, const char* what) {
  if (e == cudaErrorNotSupported)
    return fail(QCAU_ERR_UNSUPPORTED, std::string(what) + ": shape not supported by any kernel");
  return fail(QCAU_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define QCAU_CHECK_ARG(cond, msg)                          \
  do {                                                     \
    if (!(cond)) return fail(QCAU_ERR_INVALID, (msg));     \
  } while (0)

#define QCAU_CHECK_CUDA(expr)                              \
  do {                                                     \
    cudaError_t e_ = (expr);                               \
    if (e_ != cudaSuccess) return fail_cuda(e_, #expr);    \
  } while (0)

// ---------------------------------------------------------------- device error word

__device__ int g_qcau_device_error;

namespace qcau {

// The address is resolved once per device and kept for the life of the
// process (a reset of the device's primary context is not supported).
int* device_error_word() {
  static std::mutex mu;
  static std::atomic<int*> addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* a = addr[dev].load(std::memory_order_acquire);
  if (a) return a;
  std::lock_guard<std::mutex> lock(mu);
  a = addr[dev].load(std::memory_order_relaxed);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qcau_device_error) == cudaSuccess) {
      a = (int*)p;
      addr[dev].store(a, std::memory_order_release);
    }
  }
  return a;
}

// ---------------------------------------------------------------- TMA descriptors

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
               CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; i++) s[i] = strides_bytes[i];
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace qcau

// ---------------------------------------------------------------- helpers

static inline cudaStream_t to_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

namespace {

constexpr int kNumSms = 148;

// Splits of the tcgen05 two-CTA decode kernel: one CTA pair per (sequence,
// 128-head group, split), one pair per two SMs, at least 4 tiles of 128
// tokens per split.  The count minimises an estimate of the launch time
// fitted to B200 timings of 16..128 sequences x 128 heads at 32K tokens
// (within 3 % of 23 measured split counts): per wave of pairs, 12.4 us of
// setup (TMEM, barriers, the Q load, the first K tile, the partial stores)
// plus 2.39 us per tile of the longest split, each busy pair above 64
// adding 0.3 % per tile (the pairs share HBM and L2); the combine adds
// 0.015 us per partial row.  A part-filled single wave therefore beats
// more, shorter splits: 64 sequences run fastest unsplit.  With more units
// than pairs the kernel runs one pair per slot looping over units, which
// halves the setup of the later units (128 sequences x 4 splits: 1.30 ms
// against 1.34 ms); the estimate keeps the per-wave form, whose choices
// were measured best for 16, 32, 64 and 128 sequences on either grid.
double sm100_launch_us(int64_t pairs, int64_t tiles, int64_t s) {
  constexpr int64_t kSlots = kNumSms / 2;
  constexpr int64_t kQuietPairs = 64;
  const double n = (double)((tiles + s - 1) / s);
  auto wave = [&](int64_t busy) {
    const double contention = busy > kQuietPairs ? 0.0081 * (double)(busy - kQuietPairs) : 0.0;
    return 12.39 + n * (2.392 + contention);
  };
  const int64_t units = pairs * s;
  double us = (double)(units / kSlots) * wave(kSlots);
  if (units % kSlots) us += wave(units % kSlots);
  if (s > 1) us += 0.015 * (double)units;
  return us;
}

int sm100_splits(int64_t b, int64_t h, int64_t max_len) {
  const int64_t pairs = b * (h / 128 > 0 ? h / 128 : 1);
  const int64_t tiles = (max_len + 127) / 128 > 0 ? (max_len + 127) / 128 : 1;
  const int64_t cap = (max_len + 511) / 512 > 0 ? (max_len + 511) / 512 : 1;
  int best = 1;
  double best_us = sm100_launch_us(pairs, tiles, 1);
  for (int s = 2; s <= 32 && s <= cap; s++) {
    const double us = sm100_launch_us(pairs, tiles, s);
    if (us < best_us - 1e-9) {
      best_us = us;
      best = s;
    }
  }
  return best;
}

// Splits of the tcgen05 gather kernel: one CTA (one per SM) per (query row,
// head group, split); the count minimises waves x (set-up + tiles of 128 rows
// per split), the set-up (TMEM, barriers, Q, the first gathers) worth about
// one and a half tiles, plus half a tile for the merge of several splits.
int gather_splits(int64_t rows, int64_t h, int64_t d_qk, int64_t max_len) {
  const int nh = gather_heads_per_cta(h, d_qk);
  const int64_t ctas = rows * ((h + nh - 1) / nh);
  const int64_t tiles = max_len > 0 ? (max_len + 127) / 128 : 1;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= 64 && s <= tiles; s++) {
    const int64_t units = ctas * s;
    const double waves = (double)((units + kNumSms - 1) / kNumSms);
    const double cost = waves * (1.5 + (double)((tiles + s - 1) / s)) + (s > 1 ? 0.5 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

// Gathered-row attention on the tcgen05 gather kernel; a shape or device it
// does not take is an error (there is no other path).
cudaError_t run_gather(const AttnArgs& a, cudaStream_t st) {
  return launch_attn_gather_sm100(a, st);
}

// Balanced decode schedule of the pair kernel (one query token per
// sequence): the tiles of every (row, 128-head group) at max_len, row after
// row, are cut into one equal range per CTA pair (74 on B200; small batches
// keep the split count, see below).  A pair runs its range as pieces cut at row
// ends, so no pair idles and none runs more than a few pieces; a row cut
// into several pieces gets one partial slot per piece.  `splits` is the most
// pieces of any row (the owner of tile x is the largest q with
// floor(q G / P) <= x, as in the kernel).
struct StreamPlan {
  int64_t nt = 0, pairs = 0;
  int splits = 0;  // 0: not applicable
};

StreamPlan sm100_stream_plan(int64_t rows, int64_t h, int64_t max_len) {
  StreamPlan sp;
  const int64_t hgroups = h >= 128 ? h / 128 : 1;
  const int64_t nt = (max_len + 127) / 128;
  const int64_t v = rows * hgroups;
  if (v <= 0 || nt <= 0) return sp;
  const int64_t g = v * nt;
  int64_t pairs = kNumSms / 2;
  if (pairs > g / 4) pairs = g / 4;
  if (pairs < 1) pairs = 1;
  // the plan's set-up and merge have to pay for themselves: under 32 tiles
  // a pair they do not (32 x 4096 at 128 heads: 63.5 against 60.1 us), nor
  // under 64 where the split count would run unsplit, with no merge at all
  // (128 x 4096: 179 against 173 us; 64 x 32768, 221 tiles a pair: 0.697
  // against 0.764 ms; 16 x 32768, split anyway: 164 against 171 us)
  if (g < 32 * pairs || (sm100_splits(rows, h, max_len) <= 1 && g < 64 * pairs)) return sp;
  int64_t most = 1;
  for (int64_t i = 0; i < v; i++) {
    const int64_t first = ((i * nt + 1) * pairs - 1) / g;
    const int64_t last = ((i + 1) * nt * pairs - 1) / g;
    if (last - first + 1 > most) most = last - first + 1;
  }
  sp.nt = nt;
  sp.pairs = pairs;
  sp.splits = (int)most;
  return sp;
}

size_t attn_ws_bytes(int64_t rows, int64_t h, int64_t d_v, int splits) {
  if (splits <= 1) return 0;
  return align256((size_t)rows * splits * h * d_v * 4) + align256((size_t)rows * splits * h * 2 * 4);
}

// Workspace of run_decode_attn for `rows` query tokens.  Head counts that
// the two-CTA kernel takes (with 576-wide keys and 64-token pages) are sized
// for its split count; the gather kernel, which runs the other shapes, caps
// its split count to the same size.
size_t decode_ws_bytes(int64_t rows, int64_t h, int64_t d_v, int64_t max_len, int64_t qlen) {
  const bool pair_heads = d_v == 512 && (h % 128 == 0 || h == 64 || h == 32 || h == 16);
  if (pair_heads) {
    // decode rows (qlen 1) may take the balanced schedule's slots
    const StreamPlan sp = qlen == 1 ? sm100_stream_plan(rows, h, max_len) : StreamPlan{};
    const int rule = sm100_splits(rows, h, max_len);
    return attn_ws_bytes(rows, h, d_v, sp.splits > rule ? sp.splits : rule);
  }
  return attn_ws_bytes(rows, h, d_v,
                       std::max(gather_splits(rows, h, 576, max_len),
                                gather_splits(rows, h, 512, max_len)));
}

// Runs paged attention for a.b sequences x a.s query tokens (s = 1: decode;
// s > 1: token t sees the prefix up to its own position) with partials in
// `ws` when the KV range is split (its size, decode_ws_bytes, checked by the
// caller).
int run_decode_attn(AttnArgs a, void* ws, cudaStream_t st) {
  const bool sm100 = decode_attn_sm100_supported(a);
  const int64_t rows = a.b * a.s;
  // decode rows of the pair kernel take the balanced schedule when their
  // lengths fill it (the kernel checks), else the split count; the partial
  // slots cover both.  Prefill rows and fixed split ranges take the split
  // count; the gather kernel its own count, within the same workspace.
  StreamPlan sp;
  if (sm100 && a.s == 1 && a.splits_total <= 0 && !a.peer)
    sp = sm100_stream_plan(rows, a.h, a.max_len);
  if (sp.splits > 0) {
    const int rule = sm100_splits(rows, a.h, a.max_len);
    a.stream = 1;
    a.stream_nt = sp.nt;
    a.stream_pairs = sp.pairs;
    a.stream_usplits = rule;  // the fall-back for batches that do not fill the plan
    a.splits = sp.splits > rule ? sp.splits : rule;
  } else if (sm100) {
    a.splits = sm100_splits(rows, a.h, a.max_len);
  } else {
    a.splits = gather_splits(rows, a.h, a.d_qk, a.max_len);
    const size_t room = decode_ws_bytes(rows, a.h, a.d_v, a.max_len, a.s);
    while (a.splits > 1 && attn_ws_bytes(rows, a.h, a.d_v, a.splits) > room) a.splits--;
  }
  const bool partials = a.splits > 1;
  if (partials) {
    // the pair kernel keeps its O partials as O / l in fp16 (half the bytes
    // written and merged; the workspace is sized for fp32, the gather
    // kernel's format)
    a.part_f16 = sm100 ? 1 : 0;
    a.part_o = reinterpret_cast<float*>(ws);
    a.part_ml = reinterpret_cast<float*>(
        reinterpret_cast<uint8_t*>(ws) +
        align256((size_t)rows * a.splits * a.h * a.d_v * (a.part_f16 ? 2 : 4)));
  }
  if (sm100) {
    QCAU_CHECK_CUDA(launch_decode_attn_sm100(a, st));
  } else {
    QCAU_CHECK_CUDA(run_gather(a, st));
  }
  if (partials) QCAU_CHECK_CUDA(launch_attn_combine(a, st));
  return QCAU_OK;
}

}  // namespace

// ---------------------------------------------------------------- ABI

extern "C" {

int qcau_version(void) { return 100; }

const char* qcau_last_error(void) { return g_last_error.c_str(); }

int qcau_device_error(void* stream) {
  QCAU_CHECK_CUDA(cudaStreamSynchronize(to_stream(stream)));
  int v = 0;
  QCAU_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_qcau_device_error, sizeof(int)));
  if (v) {
    const int zero = 0;
    QCAU_CHECK_CUDA(cudaMemcpyToSymbol(g_qcau_device_error, &zero, sizeof(int)));
  }
  return v;
}

int qcau_act_quant(const void* x, void* y, void* s, int64_t m, int64_t n, int32_t block_size,
                   int32_t round_scale, int32_t scale_dtype, int32_t inplace, void* stream) {
  QCAU_CHECK_ARG(x != nullptr, "act_quant: x is NULL");
  QCAU_CHECK_ARG(m >= 0 && n > 0, "act_quant: bad shape");
  QCAU_CHECK_ARG(block_size == 32 || block_size == 64 || block_size == 128 || block_size == 256,
                 "act_quant: block_size must be 32, 64, 128 or 256");
  QCAU_CHECK_ARG(n % block_size == 0, "act_quant: last dimension must be divisible by block_size");
  QCAU_CHECK_ARG(scale_dtype == QCAU_SCALE_F32 || scale_dtype == QCAU_SCALE_E8M0,
                 "act_quant: bad scale dtype");
  QCAU_CHECK_ARG(scale_dtype == QCAU_SCALE_F32 || round_scale,
                 "act_quant: E8M0 scales require round_scale (scale_fmt='ue8m0')");
  QCAU_CHECK_ARG(inplace || (y != nullptr && s != nullptr), "act_quant: y/s are NULL");
  QCAU_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "act_quant: x must be 16-byte aligned");
  QCAU_CHECK_CUDA(launch_act_quant(x, y, s, m, n, block_size, round_scale,
                                   scale_dtype == QCAU_SCALE_E8M0, inplace, to_stream(stream)));
  return QCAU_OK;
}

int qcau_fp8_gemm(const void* a, const void* a_s, const void* b, const void* b_s, void* c,
                  int64_t m, int64_t n, int64_t k, int32_t scale_dtype, int32_t out_dtype,
                  void* stream) {
  QCAU_CHECK_ARG(a && a_s && b && b_s && c, "fp8_gemm: NULL pointer");
  QCAU_CHECK_ARG(m >= 0 && n > 0 && k > 0, "fp8_gemm: bad shape");
  QCAU_CHECK_ARG(k % 128 == 0, "fp8_gemm: K must be a multiple of 128");
  QCAU_CHECK_ARG(n % 128 == 0, "fp8_gemm: N must be a multiple of 128");
  QCAU_CHECK_ARG(scale_dtype == QCAU_SCALE_F32 || scale_dtype == QCAU_SCALE_E8M0,
                 "fp8_gemm: bad scale dtype");
  QCAU_CHECK_ARG(out_dtype == QCAU_OUT_BF16 || out_dtype == QCAU_OUT_F32, "fp8_gemm: bad out dtype");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                   reinterpret_cast<uintptr_t>(c)) & 15) == 0,
                 "fp8_gemm: operands must be 16-byte aligned");
  const int e8 = scale_dtype == QCAU_SCALE_E8M0;
  QCAU_CHECK_CUDA(launch_fp8_gemm(a, a_s, b, b_s, c, m, n, k, e8, e8, out_dtype == QCAU_OUT_F32,
                                  to_stream(stream)));
  return QCAU_OK;
}

int qcau_head_norm_rope(void* q, const void* gamma, const float* freqs, int64_t b, int64_t s,
                        int64_t h, int64_t d, int64_t row_stride, int64_t rope_dim, int64_t npos,
                        int64_t pos0, float eps, int32_t do_norm, void* stream) {
  QCAU_CHECK_ARG(q != nullptr, "head_norm_rope: q is NULL");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h >= 0 && d > 0 && d <= 1024 && d % 2 == 0,
                 "head_norm_rope: bad shape");
  QCAU_CHECK_ARG(rope_dim >= 0 && rope_dim % 2 == 0 && rope_dim <= d,
                 "head_norm_rope: rope_dim must be even and <= head_dim");
  QCAU_CHECK_ARG(rope_dim == 0 || (freqs != nullptr && pos0 >= 0 && pos0 + s <= npos),
                 "head_norm_rope: freqs_cis does not cover the query positions");
  QCAU_CHECK_ARG(row_stride >= d && row_stride % 2 == 0, "head_norm_rope: bad row stride");
  QCAU_CHECK_CUDA(launch_head_norm_rope(q, gamma, freqs, nullptr, b, s, h, (int)d, row_stride,
                                        (int)rope_dim, pos0, eps, do_norm, rope_dim > 0, 0,
                                        to_stream(stream)));
  return QCAU_OK;
}

int qcau_rope(void* x, const float* freqs, int64_t b, int64_t s, int64_t h, int64_t d,
              int64_t row_stride, int64_t rope_dim, int64_t npos, int64_t pos0, int32_t inverse,
              void* stream) {
  QCAU_CHECK_ARG(x != nullptr && freqs != nullptr, "rope: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h >= 0 && d > 0 && d <= 1024 && d % 2 == 0, "rope: bad shape");
  QCAU_CHECK_ARG(rope_dim > 0 && rope_dim % 2 == 0 && rope_dim <= d,
                 "rope: rope_dim must be even and <= head_dim");
  QCAU_CHECK_ARG(pos0 >= 0 && pos0 + s <= npos, "rope: freqs_cis does not cover the positions");
  QCAU_CHECK_ARG(row_stride >= d && row_stride % 2 == 0, "rope: bad row stride");
  QCAU_CHECK_CUDA(launch_head_norm_rope(x, nullptr, freqs, nullptr, b, s, h, (int)d, row_stride,
                                        (int)rope_dim, pos0, 0.f, 0, 1, inverse,
                                        to_stream(stream)));
  return QCAU_OK;
}

static int check_attn_widths(int64_t d_qk, int64_t d_v, int64_t d_kv, const char* who) {
  if (!((d_qk == 512 && d_v == 512) || (d_qk == 576 && d_v == 512)))
    return fail(QCAU_ERR_UNSUPPORTED,
                std::string(who) + ": supported (d_qk, d_v) are (512, 512) and (576, 512)");
  if (d_kv < d_qk || d_kv % 8 != 0)
    return fail(QCAU_ERR_INVALID, std::string(who) + ": kv row width must be >= d_qk and a multiple of 8");
  return QCAU_OK;
}

int qcau_sparse_attn(const void* q, const void* kv, const float* attn_sink,
                     const int32_t* topk_idxs, void* o, int64_t b, int64_t s, int64_t h,
                     int64_t d_qk, int64_t d_v, int64_t d_kv, int64_t n_kv, int64_t topk,
                     float softmax_scale, int32_t inv_rope, const float* freqs, int64_t rope_dim,
                     int64_t npos, int64_t pos0, void* stream) {
  QCAU_CHECK_ARG(q && kv && topk_idxs && o, "sparse_attn: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h > 0 && topk >= 0, "sparse_attn: bad shape");
  QCAU_CHECK_ARG(n_kv > 0, "sparse_attn: kv must contain at least one latent row");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "sparse_attn");
  if (rc) return rc;
  if (inv_rope) {
    QCAU_CHECK_ARG(freqs != nullptr && rope_dim > 0 && rope_dim % 4 == 0 && rope_dim <= d_v,
                   "sparse_attn: bad inverse-RoPE arguments");
    QCAU_CHECK_ARG(pos0 >= 0 && pos0 + s <= npos, "sparse_attn: freqs_cis does not cover the positions");
  }
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d_qk;
  a.kv = kv;
  a.idx = topk_idxs;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = s; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv; a.n_kv = n_kv;
  a.topk = topk;
  a.max_len = topk;
  a.splits = 1;
  a.scale = softmax_scale;
  a.freqs = freqs;
  a.inv_rope = inv_rope;
  a.rope_dim = (int)rope_dim;
  a.pos0 = pos0;
  QCAU_CHECK_CUDA(run_gather(a, to_stream(stream)));
  return QCAU_OK;
}

size_t qcau_forward_workspace_size(int64_t b, int64_t s, int64_t h, int64_t d, int64_t dc) {
  const size_t rows = (size_t)(b * s);
  return align256(rows * dc) + align256(rows * (dc / 128) * 4) + align256(rows * h * d * 2);
}

int qcau_forward(const void* c_q, const void* wq_b, const void* wq_b_scale, int32_t w_scale_dtype,
                 int32_t act_round_scale, const void* gamma, const void* kv,
                 const int32_t* topk_idxs, const float* attn_sink, const float* freqs, void* o,
                 int64_t b, int64_t s, int64_t h, int64_t d, int64_t dc, int64_t n_kv,
                 int64_t topk, int64_t rope_dim, int64_t npos, int64_t pos0, float norm_eps,
                 float softmax_scale, void* workspace, size_t workspace_bytes, void* stream) {
  QCAU_CHECK_ARG(c_q && wq_b && wq_b_scale && kv && topk_idxs && freqs && o,
                 "qcau_forward: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h > 0 && d > 0 && dc > 0, "qcau_forward: bad shape");
  QCAU_CHECK_ARG(dc % 128 == 0, "qcau_forward: D_C must be a multiple of 128");
  QCAU_CHECK_ARG((h * d) % 128 == 0, "qcau_forward: H*Dh must be a multiple of 128");
  QCAU_CHECK_ARG(n_kv > 0, "qcau_forward: kv must contain at least one latent row");
  QCAU_CHECK_ARG(rope_dim > 0 && rope_dim % 4 == 0 && rope_dim <= d, "qcau_forward: bad rope_dim");
  QCAU_CHECK_ARG(pos0 >= 0 && pos0 + s <= npos, "qcau_forward: freqs_cis does not cover the positions");
  QCAU_CHECK_ARG(w_scale_dtype == QCAU_SCALE_F32 || w_scale_dtype == QCAU_SCALE_E8M0,
                 "qcau_forward: bad scale dtype");
  int rc = check_attn_widths(d, d, d, "qcau_forward");
  if (rc) return rc;
  const size_t need = qcau_forward_workspace_size(b, s, h, d, dc);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE, "qcau_forward: workspace too small (need " +
                                        std::to_string(need) + " bytes)");
  if (b * s == 0) return QCAU_OK;
  cudaStream_t st = to_stream(stream);
  const int64_t rows = b * s;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  uint8_t* xq = ws;
  void* sq = ws + align256(rows * dc);
  void* q = ws + align256(rows * dc) + align256(rows * (dc / 128) * 4);
  const int a_e8 = act_round_scale ? 1 : 0;
  QCAU_CHECK_CUDA(launch_act_quant(c_q, xq, sq, rows, dc, 128, act_round_scale, a_e8, 0, st));
  QCAU_CHECK_CUDA(launch_fp8_gemm(xq, sq, wq_b, wq_b_scale, q, rows, h * d, dc, a_e8,
                                  w_scale_dtype == QCAU_SCALE_E8M0, 0, st));
  QCAU_CHECK_CUDA(launch_head_norm_rope(q, gamma, freqs, nullptr, b, s, h, (int)d, d,
                                        (int)rope_dim, pos0, norm_eps, 1, 1, 0, st));
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d;
  a.kv = kv;
  a.idx = topk_idxs;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = s; a.h = h; a.d_qk = d; a.d_v = d; a.d_kv = d; a.n_kv = n_kv; a.topk = topk;
  a.max_len = topk;
  a.splits = 1;
  a.scale = softmax_scale;
  a.freqs = freqs;
  a.inv_rope = 1;
  a.rope_dim = (int)rope_dim;
  a.pos0 = pos0;
  QCAU_CHECK_CUDA(run_gather(a, st));
  return QCAU_OK;
}

size_t qcau_decode_attn_workspace_size(int64_t b, int64_t h, int64_t d_v, int64_t max_seqlen) {
  return decode_ws_bytes(b, h, d_v, max_seqlen, 1);
}

int qcau_decode_attn_paged(const void* q, const void* cache, const int32_t* block_table,
                           const int32_t* seqlens, const float* attn_sink, void* o, int64_t b,
                           int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv, int64_t page_size,
                           int64_t max_pages, int64_t num_pages, int64_t max_seqlen,
                           float softmax_scale, void* workspace, size_t workspace_bytes,
                           void* stream) {
  QCAU_CHECK_ARG(q && cache && block_table && seqlens && o, "decode_attn_paged: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "decode_attn_paged: bad shape");
  QCAU_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= max_pages * page_size,
                 "decode_attn_paged: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "decode_attn_paged");
  if (rc) return rc;
  const size_t need = qcau_decode_attn_workspace_size(b, h, d_v, max_seqlen);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE, "decode_attn_paged: workspace too small (need " +
                                        std::to_string(need) + " bytes)");
  if (b == 0) return QCAU_OK;
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d_qk;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = 1; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  return run_decode_attn(a, workspace, to_stream(stream));
}

int qcau_decode_attn_paged_blocked(const void* q, int64_t q_hblock, const void* cache,
                                   const int32_t* block_table, const int32_t* seqlens,
                                   const float* attn_sink, void* o, int64_t o_hblock, int64_t b,
                                   int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                                   int64_t page_size, int64_t max_pages, int64_t num_pages,
                                   int64_t max_seqlen, float softmax_scale, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  QCAU_CHECK_ARG(q && cache && block_table && seqlens && o,
                 "decode_attn_paged_blocked: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "decode_attn_paged_blocked: bad shape");
  QCAU_CHECK_ARG(q_hblock > 0 && o_hblock > 0 && h % q_hblock == 0 && h % o_hblock == 0,
                 "decode_attn_paged_blocked: head blocks must divide h");
  QCAU_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= max_pages * page_size,
                 "decode_attn_paged_blocked: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "decode_attn_paged_blocked");
  if (rc) return rc;
  const size_t need = qcau_decode_attn_workspace_size(b, h, d_v, max_seqlen);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE, "decode_attn_paged_blocked: workspace too small (need " +
                                        std::to_string(need) + " bytes)");
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d_qk;
  a.q_hblock = q_hblock;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.sink = attn_sink;
  a.o = o;
  a.o_hblock = o_hblock;
  a.b = b; a.s = 1; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  if (!decode_attn_sm100_supported(a))
    return fail(QCAU_ERR_UNSUPPORTED,
                "decode_attn_paged_blocked: needs the sm_100a pair kernel (d_qk 576, d_v 512, "
                "page 64, h a multiple of 128, head blocks a multiple of 64 or 8, 16 or 32)");
  if (b == 0) return QCAU_OK;
  return run_decode_attn(a, workspace, to_stream(stream));
}

size_t qcau_sparse_attn_fp8_workspace_size(int64_t b, int64_t s, int64_t h, int64_t topk) {
  return attn_ws_bytes(b * s, h, 512, gather_splits(b * s, h, 576, topk));
}

int qcau_sparse_attn_fp8(const void* q, const void* kv_latent, const float* kv_scale,
                         const void* kv_rope, const float* attn_sink, const int32_t* topk_idxs,
                         void* o, int64_t b, int64_t s, int64_t h, int64_t n_kv, int64_t topk,
                         float softmax_scale, void* workspace, size_t workspace_bytes,
                         void* stream) {
  QCAU_CHECK_ARG(q && kv_latent && kv_scale && kv_rope && topk_idxs && o,
                 "sparse_attn_fp8: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h > 0 && topk > 0, "sparse_attn_fp8: bad shape");
  QCAU_CHECK_ARG(n_kv > 0, "sparse_attn_fp8: kv must contain at least one latent row");
  QCAU_CHECK_ARG((reinterpret_cast<uintptr_t>(kv_latent) & 31) == 0 &&
                     (reinterpret_cast<uintptr_t>(kv_rope) & 15) == 0,
                 "sparse_attn_fp8: kv_latent must be 32-byte and kv_rope 16-byte aligned");
  const size_t need = qcau_sparse_attn_fp8_workspace_size(b, s, h, topk);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE, "sparse_attn_fp8: workspace too small (need " +
                                        std::to_string(need) + " bytes)");
  if (b == 0 || s == 0) return QCAU_OK;
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = 576;
  a.idx = topk_idxs;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = s; a.h = h; a.d_qk = 576; a.d_v = 512; a.d_kv = 576;
  a.n_kv = n_kv;
  a.topk = topk;
  a.max_len = topk;
  a.scale = softmax_scale;
  a.kv_fp8 = reinterpret_cast<const uint8_t*>(kv_latent);
  a.kv_scale = kv_scale;
  a.kv_rope = kv_rope;
  a.kv = kv_latent;
  cudaStream_t st = to_stream(stream);
  a.splits = gather_splits(b * s, h, 576, topk);
  if (a.splits > 1) {
    a.part_o = reinterpret_cast<float*>(workspace);
    a.part_ml = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) +
                                         align256((size_t)b * s * a.splits * h * 512 * 4));
  }
  QCAU_CHECK_CUDA(run_gather(a, st));
  if (a.splits > 1) QCAU_CHECK_CUDA(launch_attn_combine(a, st));
  return QCAU_OK;
}

size_t qcau_prefill_attn_workspace_size(int64_t b, int64_t s, int64_t h, int64_t d_v,
                                        int64_t max_seqlen) {
  return decode_ws_bytes(b * s, h, d_v, max_seqlen, s);
}

int qcau_prefill_attn_paged(const void* q, const void* cache, const int32_t* block_table,
                            const int32_t* seqlens, const float* attn_sink, void* o, int64_t b,
                            int64_t s, int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                            int64_t page_size, int64_t max_pages, int64_t num_pages,
                            int64_t max_seqlen, float softmax_scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
  QCAU_CHECK_ARG(q && cache && block_table && seqlens && o, "prefill_attn_paged: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 1 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "prefill_attn_paged: bad shape");
  QCAU_CHECK_ARG(max_seqlen >= s, "prefill_attn_paged: max_seqlen must cover the s new tokens");
  QCAU_CHECK_ARG(max_seqlen <= max_pages * page_size,
                 "prefill_attn_paged: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "prefill_attn_paged");
  if (rc) return rc;
  const size_t need = qcau_prefill_attn_workspace_size(b, s, h, d_v, max_seqlen);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE, "prefill_attn_paged: workspace too small (need " +
                                        std::to_string(need) + " bytes)");
  if (b == 0) return QCAU_OK;
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d_qk;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = s; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  return run_decode_attn(a, workspace, to_stream(stream));
}

}  // extern "C"

// ---------------------------------------------------------------- no-alloc decode scratch

// Split-KV partials of qcau_decode_attn_paged_noalloc.  Module-scope device
// storage: each device that loads the library holds it until the process exits.
static __device__ __align__(256) uint8_t g_decode_scratch[QCAU_DECODE_STATIC_SCRATCH_BYTES];

// Address of g_decode_scratch on the current device, resolved once per device
// with that device current and kept for the life of the process (a reset of
// the device's primary context is not supported).
static int decode_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  QCAU_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    return fail(QCAU_ERR_UNSUPPORTED, "decode_attn_paged_noalloc: device ordinal above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    QCAU_CHECK_CUDA(cudaGetSymbolAddress(&p, g_decode_scratch));
    addr[dev] = p;
  }
  *out = addr[dev];
  return QCAU_OK;
}

extern "C" {

int qcau_decode_attn_paged_noalloc(const void* q, const void* cache, const int32_t* block_table,
                                   const int32_t* seqlens, const float* attn_sink, void* o,
                                   int64_t b, int64_t h, int64_t d_qk, int64_t d_v, int64_t d_kv,
                                   int64_t page_size, int64_t max_pages, int64_t num_pages,
                                   int64_t max_seqlen, float softmax_scale, void* stream) {
  QCAU_CHECK_ARG(q && cache && block_table && seqlens && o,
                 "decode_attn_paged_noalloc: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "decode_attn_paged_noalloc: bad shape");
  QCAU_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= max_pages * page_size,
                 "decode_attn_paged_noalloc: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "decode_attn_paged_noalloc");
  if (rc) return rc;
  const size_t need = qcau_decode_attn_workspace_size(b, h, d_v, max_seqlen);
  if (need > QCAU_DECODE_STATIC_SCRATCH_BYTES)
    return fail(QCAU_ERR_WORKSPACE,
                "decode_attn_paged_noalloc: split-KV partials need " + std::to_string(need) +
                    " bytes, more than the " +
                    std::to_string((size_t)QCAU_DECODE_STATIC_SCRATCH_BYTES) +
                    "-byte static scratch; use qcau_decode_attn_paged with a workspace");
  if (b == 0) return QCAU_OK;
  void* scratch = nullptr;
  rc = decode_scratch_address(&scratch);
  if (rc) return rc;
  AttnArgs a{};
  a.q = q;
  a.q_row_stride = d_qk;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = 1; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  return run_decode_attn(a, scratch, to_stream(stream));
}

int qcau_dequant_fp8_weight(const void* w, const void* w_scale, int32_t scale_dtype, void* out_bf16,
                            int64_t rows, int64_t cols, void* stream) {
  QCAU_CHECK_ARG(w && w_scale && out_bf16, "dequant_fp8_weight: NULL pointer");
  QCAU_CHECK_ARG(rows >= 0 && cols >= 0, "dequant_fp8_weight: bad shape");
  QCAU_CHECK_ARG(scale_dtype == QCAU_SCALE_F32 || scale_dtype == QCAU_SCALE_E8M0,
                 "dequant_fp8_weight: bad scale dtype");
  QCAU_CHECK_CUDA(launch_dequant_fp8_weight(w, w_scale, scale_dtype == QCAU_SCALE_E8M0, out_bf16,
                                            rows, cols, to_stream(stream)));
  return QCAU_OK;
}

size_t qcau_gopu_workspace_size(int64_t rows, int64_t groups, int64_t rank_dim) {
  const int64_t k2 = groups * rank_dim;
  return align256((size_t)(rows * k2 * 2)) + align256((size_t)(rows * k2)) +
         align256((size_t)(rows * (k2 / 128) * 4));
}

int qcau_gopu(const void* o, const void* wo_a, const void* wo_b, const void* wo_b_scale,
              int32_t scale_dtype, int32_t act_round_scale, void* y, int32_t out_dtype,
              int64_t rows, int64_t groups, int64_t group_dim, int64_t rank_dim, int64_t dim,
              void* workspace, size_t workspace_bytes, void* stream) {
  QCAU_CHECK_ARG(o && wo_a && wo_b && wo_b_scale && y, "gopu: NULL pointer");
  QCAU_CHECK_ARG(rows >= 0 && groups > 0 && group_dim > 0 && rank_dim > 0 && dim > 0,
                 "gopu: bad shape");
  QCAU_CHECK_ARG(group_dim % 64 == 0, "gopu: the group width must be a multiple of 64");
  QCAU_CHECK_ARG(rank_dim % 128 == 0, "gopu: o_lora_rank must be a multiple of 128");
  QCAU_CHECK_ARG(dim % 128 == 0, "gopu: the output width must be a multiple of 128");
  QCAU_CHECK_ARG(scale_dtype == QCAU_SCALE_F32 || scale_dtype == QCAU_SCALE_E8M0,
                 "gopu: bad scale dtype");
  QCAU_CHECK_ARG(out_dtype == QCAU_OUT_BF16 || out_dtype == QCAU_OUT_F32, "gopu: bad out dtype");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(wo_a) |
                   reinterpret_cast<uintptr_t>(wo_b) | reinterpret_cast<uintptr_t>(y)) & 15) == 0,
                 "gopu: operands must be 16-byte aligned");
  const size_t need = qcau_gopu_workspace_size(rows, groups, rank_dim);
  if (workspace_bytes < need || (need && !workspace))
    return fail(QCAU_ERR_WORKSPACE,
                "gopu: workspace too small (need " + std::to_string(need) + " bytes)");
  if (rows == 0) return QCAU_OK;
  cudaStream_t st = to_stream(stream);
  const int64_t k2 = groups * rank_dim;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  void* h = ws;                                        // [rows, groups, rank_dim] bf16
  void* xq = ws + align256((size_t)(rows * k2 * 2));  // its FP8 codes
  void* sq = reinterpret_cast<uint8_t*>(xq) + align256((size_t)(rows * k2));
  // wo_a: h[r, g, :] = o[r, g, :] . wo_a[g]^T  (model.py:537-541, bf16 einsum)
  BmmArgs b{};
  b.a = o;
  b.a_bstride = group_dim;
  b.a_rstride = groups * group_dim;
  b.b = wo_a;
  b.b_bstride = rank_dim * group_dim;
  b.b_rstride = group_dim;
  b.b_kmajor = 1;
  b.c = h;
  b.c_bstride = rank_dim;
  b.c_rstride = k2;
  b.batch = groups;
  b.m = rows;
  b.n = rank_dim;
  b.k = group_dim;
  QCAU_CHECK_CUDA(launch_bf16_bmm(b, st));
  // wo_b: linear() -> act_quant + fp8_gemm (model.py:108-120, 166-180)
  const int a_e8 = act_round_scale ? 1 : 0;
  QCAU_CHECK_CUDA(launch_act_quant(h, xq, sq, rows, k2, 128, act_round_scale, a_e8, 0, st));
  QCAU_CHECK_CUDA(launch_fp8_gemm(xq, sq, wo_b, wo_b_scale, y, rows, dim, k2, a_e8,
                                  scale_dtype == QCAU_SCALE_E8M0, out_dtype == QCAU_OUT_F32, st));
  return QCAU_OK;
}

int qcau_rotate_fp4(void* x, int64_t rows, int64_t d, int32_t hadamard, int32_t fp4,
                    void* stream) {
  QCAU_CHECK_ARG(x != nullptr, "rotate_fp4: x is NULL");
  QCAU_CHECK_ARG(rows >= 0 && d == 128, "rotate_fp4: rows of 128 values are supported");
  QCAU_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 7) == 0, "rotate_fp4: x must be 8-byte aligned");
  QCAU_CHECK_CUDA(launch_rotate_fp4(x, rows, hadamard ? 1 : 0, fp4 ? 1 : 0, to_stream(stream)));
  return QCAU_OK;
}

static int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

size_t qcau_indexer_scores_workspace_size(int64_t, int64_t, int64_t, int64_t) { return 0; }

size_t qcau_indexer_topk_workspace_size(int64_t b, int64_t s, int64_t h, int64_t t) {
  (void)h;
  return align256((size_t)(b * s * (t > 0 ? t : 0) * 4));
}

int qcau_indexer_raw_scores(const void* q, const void* kv, void* raw, int64_t b, int64_t s,
                            int64_t h, int64_t d, int64_t t, int64_t kv_rows, void* stream) {
  QCAU_CHECK_ARG(q && kv && raw, "indexer_raw_scores: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h > 0 && t >= 0 && kv_rows >= t,
                 "indexer_raw_scores: bad shape");
  QCAU_CHECK_ARG(d % 64 == 0 && d > 0, "indexer_raw_scores: head_dim must be a multiple of 64");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv) |
                   reinterpret_cast<uintptr_t>(raw)) & 15) == 0,
                 "indexer_raw_scores: q, kv and raw must be 16-byte aligned");
  if (b * s == 0 || t == 0) return QCAU_OK;
  const int64_t tp = round_up(t, 128);
  // raw[b, (s, h), u] = q[b, s, h, :] . kv[b, u, :], the bf16 einsum
  // (model.py:518); the B tensor map holds the t rows that exist, the rest of
  // the last 128-row tile reads as zeros
  BmmArgs m{};
  m.a = q;
  m.a_bstride = s * h * d;
  m.a_rstride = d;
  m.b = kv;
  m.b_bstride = kv_rows * d;
  m.b_rstride = d;
  m.b_kmajor = 1;
  m.b_rows = t;
  m.c = raw;
  m.c_bstride = s * h * tp;
  m.c_rstride = tp;
  m.batch = b;
  m.m = s * h;
  m.n = tp;
  m.k = d;
  QCAU_CHECK_CUDA(launch_bf16_bmm(m, to_stream(stream)));
  return QCAU_OK;
}

int qcau_indexer_scores(const void* q, const void* kv, const void* weights, float* score,
                        int64_t b, int64_t s, int64_t h, int64_t d, int64_t t, int64_t kv_rows,
                        void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  QCAU_CHECK_ARG(q && kv && weights && score, "indexer_scores: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && s >= 0 && h > 0 && h <= 128 && t >= 0 && kv_rows >= t,
                 "indexer_scores: bad shape (up to 128 heads a rank)");
  QCAU_CHECK_ARG(d == 128, "indexer_scores: index_head_dim 128 is supported");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv)) & 15) == 0,
                 "indexer_scores: q and kv must be 16-byte aligned");
  QCAU_CHECK_ARG((b * s * h) < (int64_t(1) << 31) && t < (int64_t(1) << 31),
                 "indexer_scores: too many query heads or keys");
  if (b * s == 0 || t == 0) return QCAU_OK;
  QCAU_CHECK_CUDA(launch_indexer_score_sm100(q, kv, weights, score, b, s, h, t, kv_rows,
                                             to_stream(stream)));
  return QCAU_OK;
}

int qcau_topk(const float* score, int32_t* topk_idxs, int64_t rows, int64_t t, int64_t k,
              int64_t seqlen, int64_t mask_ratio, int64_t offset, void* stream) {
  QCAU_CHECK_ARG((score || rows * t == 0) && (topk_idxs || rows * k == 0), "topk: NULL pointer");
  QCAU_CHECK_ARG(rows >= 0 && t >= 0 && k >= 0 && k <= 2048, "topk: k up to 2048 is supported");
  QCAU_CHECK_ARG(mask_ratio >= 0 && (mask_ratio == 0 || seqlen > 0),
                 "topk: the prefill mask needs seqlen");
  QCAU_CHECK_CUDA(launch_topk(score, rows, t, (int)k, topk_idxs, offset, seqlen, (int)mask_ratio,
                              to_stream(stream)));
  return QCAU_OK;
}

int qcau_indexer_topk(const void* q, const void* kv, const void* weights, int32_t* topk_idxs,
                      int64_t b, int64_t s, int64_t h, int64_t d, int64_t t, int64_t kv_rows,
                      int64_t k, int64_t start_pos, int64_t ratio, int64_t offset,
                      void* workspace, size_t workspace_bytes, void* stream) {
  QCAU_CHECK_ARG(topk_idxs != nullptr, "indexer_topk: topk_idxs is NULL");
  QCAU_CHECK_ARG(k >= 0 && k <= 2048, "indexer_topk: index_topk up to 2048 is supported");
  QCAU_CHECK_ARG(ratio > 0 && start_pos >= 0, "indexer_topk: bad ratio or start_pos");
  const size_t need = qcau_indexer_topk_workspace_size(b, s, h, t);
  if (workspace_bytes < need || !workspace)
    return fail(QCAU_ERR_WORKSPACE,
                "indexer_topk: workspace too small (need " + std::to_string(need) + " bytes)");
  float* score = reinterpret_cast<float*>(workspace);
  const int rc = qcau_indexer_scores(q, kv, weights, score, b, s, h, d, t, kv_rows, nullptr, 0,
                                     stream);
  if (rc != QCAU_OK) return rc;
  return qcau_topk(score, topk_idxs, b * s, t, k, s, start_pos == 0 ? ratio : 0, offset, stream);
}

int qcau_index_lists(int32_t* topk_idxs, int64_t bsz, int64_t seqlen, int64_t start_pos,
                     int64_t window, int64_t ratio, int64_t offset, const int32_t* selected,
                     int64_t selected_width, void* stream) {
  QCAU_CHECK_ARG(topk_idxs != nullptr, "index_lists: output is NULL");
  QCAU_CHECK_ARG(bsz >= 0 && seqlen >= 0 && start_pos >= 0 && window > 0 && ratio >= 0,
                 "index_lists: bad arguments");
  QCAU_CHECK_ARG(start_pos == 0 || seqlen == 1, "index_lists: decode steps have one token");
  const int64_t win_w = start_pos == 0 ? (seqlen < window ? seqlen : window) : window;
  int64_t comp_w = 0;
  if (selected) {
    comp_w = selected_width;
  } else if (ratio > 0) {
    comp_w = start_pos > 0 ? (start_pos + 1) / ratio : seqlen / ratio;
  }
  QCAU_CHECK_CUDA(launch_index_lists(topk_idxs, bsz, seqlen, start_pos, (int)window,
                                     (int)(ratio > 0 ? ratio : 1), offset, (int)win_w,
                                     (int)comp_w, selected, to_stream(stream)));
  return QCAU_OK;
}

int64_t qcau_index_lists_width(int64_t seqlen, int64_t start_pos, int64_t window, int64_t ratio,
                               int64_t selected_width) {
  const int64_t win_w = start_pos == 0 ? (seqlen < window ? seqlen : window) : window;
  if (selected_width > 0) return win_w + selected_width;
  if (ratio <= 0) return win_w;
  return win_w + (start_pos > 0 ? (start_pos + 1) / ratio : seqlen / ratio);
}

int qcau_compress(const float* kv, const float* score, const float* ape, float* kv_state,
                  float* score_state, void* out, int64_t bsz, int64_t seqlen, int64_t d,
                  int64_t ratio, int32_t overlap, int64_t start_pos, void* stream) {
  QCAU_CHECK_ARG(bsz >= 0 && seqlen >= 0 && d > 0 && ratio > 0 && start_pos >= 0,
                 "compress: bad shape");
  QCAU_CHECK_ARG((overlap ? 2 : 1) * ratio <= 256, "compress: windows up to 256 entries");
  QCAU_CHECK_ARG(start_pos == 0 || seqlen == 1, "compress: decode steps have one token");
  QCAU_CHECK_ARG(bsz * seqlen == 0 || (kv && score && ape), "compress: NULL input");
  QCAU_CHECK_ARG(start_pos == 0 || (kv_state && score_state && out),
                 "compress: decode needs the state and an output row");
  QCAU_CHECK_ARG(start_pos > 0 || seqlen < ratio || out, "compress: output is NULL");
  QCAU_CHECK_ARG((kv_state == nullptr) == (score_state == nullptr),
                 "compress: kv_state and score_state go together");
  if (bsz * seqlen == 0) return QCAU_OK;
  QCAU_CHECK_CUDA(launch_compress(kv, score, ape, kv_state, score_state, out, bsz, seqlen, (int)d,
                                  (int)ratio, overlap ? 1 : 0, start_pos, to_stream(stream)));
  return QCAU_OK;
}

int qcau_kv_build(const void* kv_in, void* kv_out, int64_t rows, int64_t d,
                  const float* norm_weight, int64_t norm_dim, float eps, const float* freqs,
                  const int32_t* positions, int64_t npos, int64_t rope_dim, int64_t quant_dims,
                  int32_t round_scale, void* cache, const int32_t* cache_slots,
                  int64_t cache_rows, void* stream) {
  QCAU_CHECK_ARG(kv_in != nullptr, "kv_build: kv_in is NULL");
  QCAU_CHECK_ARG(rows >= 0 && d > 0 && d % 64 == 0 && d <= 1024,
                 "kv_build: d must be a multiple of 64 up to 1024");
  QCAU_CHECK_ARG(norm_dim >= 0 && norm_dim % 64 == 0 && norm_dim <= d,
                 "kv_build: norm_dim must be a multiple of 64 up to d");
  QCAU_CHECK_ARG(rope_dim >= 0 && rope_dim % 2 == 0 && rope_dim <= d, "kv_build: bad rope_dim");
  QCAU_CHECK_ARG(rope_dim == 0 || (freqs != nullptr && positions != nullptr && npos > 0),
                 "kv_build: RoPE needs freqs_cis and positions");
  QCAU_CHECK_ARG(quant_dims >= 0 && quant_dims % 64 == 0 && quant_dims <= d - rope_dim,
                 "kv_build: quant_dims must be a multiple of 64 below the rope values");
  QCAU_CHECK_ARG(cache == nullptr || (cache_slots != nullptr && cache_rows >= 0),
                 "kv_build: a cache needs cache_slots");
  QCAU_CHECK_ARG(kv_out != nullptr || cache != nullptr, "kv_build: no destination");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(kv_in) | reinterpret_cast<uintptr_t>(kv_out) |
                   reinterpret_cast<uintptr_t>(cache)) & 3) == 0,
                 "kv_build: rows must be 4-byte aligned");
  KvBuildArgs a{};
  a.in = kv_in;
  a.out = kv_out;
  a.rows = rows;
  a.d = d;
  a.norm_weight = norm_weight;
  a.norm_dim = (int)norm_dim;
  a.eps = eps;
  a.freqs = freqs;
  a.positions = positions;
  a.npos = npos;
  a.rope_dim = (int)rope_dim;
  a.quant_dims = (int)quant_dims;
  a.round_scale = round_scale ? 1 : 0;
  a.cache = cache;
  a.slots = cache ? cache_slots : nullptr;
  a.cache_rows = cache_rows;
  QCAU_CHECK_CUDA(launch_kv_build(a, to_stream(stream)));
  return QCAU_OK;
}

int qcau_compressor_step(const float* kv, const float* score, const float* ape, float* kv_state,
                         float* score_state, int64_t bsz, int64_t seqlen, int64_t d,
                         int64_t ratio, int32_t overlap, int64_t start_pos,
                         const float* norm_weight, float eps, const float* freqs, int64_t npos,
                         int64_t rope_dim, int32_t rotate, int32_t round_scale, void* cache,
                         int64_t cache_seq_rows, int64_t cache_offset, void* rows_out,
                         void* stream) {
  QCAU_CHECK_ARG(bsz >= 0 && seqlen >= 0 && ratio > 0 && start_pos >= 0,
                 "compressor_step: bad shape");
  QCAU_CHECK_ARG(d > 0 && d % 64 == 0 && d <= 1024 && rope_dim >= 0 && rope_dim % 2 == 0 &&
                     rope_dim <= d, "compressor_step: bad head_dim or rope_dim");
  QCAU_CHECK_ARG(rotate ? d == 128 : (d - rope_dim) % 64 == 0,
                 "compressor_step: the rotated rows must be 128 wide, the others have a "
                 "multiple of 64 values below the rope part");
  QCAU_CHECK_ARG(start_pos == 0 || seqlen == 1, "compressor_step: decode steps have one token");
  QCAU_CHECK_ARG(kv_state && score_state, "compressor_step: the state is NULL");
  QCAU_CHECK_ARG(rope_dim == 0 || (freqs && npos > 0), "compressor_step: RoPE needs freqs");
  const int64_t n = start_pos == 0 ? seqlen / ratio : ((start_pos + 1) % ratio == 0 ? 1 : 0);
  const int64_t first = start_pos == 0 ? 0 : start_pos / ratio;
  QCAU_CHECK_ARG(bsz * seqlen == 0 || (kv && score && ape), "compressor_step: NULL input");
  QCAU_CHECK_ARG(bsz * n == 0 || rows_out, "compressor_step: rows_out is NULL");
  QCAU_CHECK_ARG(cache == nullptr || (cache_seq_rows > 0 && cache_offset >= 0 &&
                                      cache_offset + first + n <= cache_seq_rows),
                 "compressor_step: the compressed rows do not fit the cache rows of a sequence");
  QCAU_CHECK_ARG(((reinterpret_cast<uintptr_t>(rows_out) | reinterpret_cast<uintptr_t>(cache)) &
                  15) == 0, "compressor_step: rows_out and cache must be 16-byte aligned");
  if (bsz * seqlen == 0) return QCAU_OK;
  cudaStream_t st = to_stream(stream);
  // pooled rows [bsz, n, d] bf16 into rows_out, then built there in place
  QCAU_CHECK_CUDA(launch_compress(kv, score, ape, kv_state, score_state, rows_out, bsz, seqlen,
                                  (int)d, (int)ratio, overlap ? 1 : 0, start_pos, st));
  if (n == 0) return QCAU_OK;
  KvBuildArgs a{};
  a.in = rows_out;
  a.out = rows_out;
  a.rows = bsz * n;
  a.d = d;
  a.norm_weight = norm_weight;
  a.norm_dim = (int)d;
  a.eps = eps;
  a.freqs = freqs;
  a.npos = npos;
  a.rope_dim = (int)rope_dim;
  a.quant_dims = rotate ? 0 : (int)(d - rope_dim);
  a.round_scale = round_scale ? 1 : 0;
  // compressed row i of sequence b: position (first + i) * ratio, cache row
  // b * cache_seq_rows + cache_offset + first + i (model.py:459-476)
  a.seq_rows = n;
  a.pos_base = first * ratio;
  a.pos_step = ratio;
  a.slot_seq_stride = cache_seq_rows;
  a.slot_base = cache_offset + first;
  if (!rotate) {
    a.cache = cache;
    a.cache_rows = cache ? bsz * cache_seq_rows : 0;
  }
  QCAU_CHECK_CUDA(launch_kv_build(a, st));
  if (rotate) {
    QCAU_CHECK_CUDA(launch_rotate_fp4(rows_out, bsz * n, 1, 1, st));
    if (cache) {
      const size_t row_bytes = (size_t)d * 2;
      QCAU_CHECK_CUDA(cudaMemcpy2DAsync(
          reinterpret_cast<uint8_t*>(cache) + (size_t)(cache_offset + first) * row_bytes,
          (size_t)cache_seq_rows * row_bytes, rows_out, (size_t)n * row_bytes,
          (size_t)n * row_bytes, (size_t)bsz, cudaMemcpyDeviceToDevice, st));
    }
  }
  return QCAU_OK;
}

// Workspace layout of the absorbed decode layer.
struct MlaWs {
  size_t xq, sq, q, qabs, olat, ov, xo, so, attn, total;
};

static MlaWs mla_ws(const qcau_mla_dims* d) {
  MlaWs w{};
  const size_t B = (size_t)d->batch, H = (size_t)d->n_heads;
  const size_t dq = (size_t)(d->d_nope + d->d_rope), dabs = (size_t)(d->kv_lora + d->d_rope);
  size_t off = 0;
  w.xq = off; off += align256(B * d->dc);
  w.sq = off; off += align256(B * (d->dc / 128) * 4);
  w.q = off; off += align256(B * H * dq * 2);
  w.qabs = off; off += align256(B * H * dabs * 2);
  w.olat = off; off += align256(B * H * d->kv_lora * 2);
  w.ov = off; off += align256(B * H * d->d_v * 2);
  w.xo = off; off += align256(B * H * d->d_v);
  w.so = off; off += align256(B * ((H * d->d_v) / 128) * 4);
  w.attn = off; off += decode_ws_bytes(d->batch, d->n_heads, d->kv_lora, d->max_seqlen, 1);
  w.total = off;
  return w;
}

size_t qcau_mla_decode_workspace_size(const qcau_mla_dims* dims) {
  return dims ? mla_ws(dims).total : 0;
}

// Checks of the layer dimensions shared by the layer entry points.
static int check_mla_dims(const qcau_mla_dims* d, const char* what) {
  const std::string w = what;
  QCAU_CHECK_ARG(d != nullptr, w + ": dims is NULL");
  QCAU_CHECK_ARG(d->batch >= 0 && d->n_heads > 0 && d->dc > 0 && d->dim > 0, w + ": bad shape");
  QCAU_CHECK_ARG(d->d_nope == 128 && d->d_rope == 64 && d->kv_lora == 512 && d->d_v == 128,
                 w + ": supported head layout is d_nope 128, d_rope 64, kv_lora 512, d_v 128");
  QCAU_CHECK_ARG(d->dc % 128 == 0 && d->dim % 128 == 0 && (d->n_heads * d->d_v) % 128 == 0 &&
                     (d->n_heads * (d->d_nope + d->d_rope)) % 128 == 0,
                 w + ": widths must be multiples of 128");
  QCAU_CHECK_ARG(d->w_scale_dtype == QCAU_SCALE_F32 || d->w_scale_dtype == QCAU_SCALE_E8M0,
                 w + ": bad scale dtype");
  return QCAU_OK;
}

// q side of the layer: q_abs [B, H, kv_lora + d_rope] bf16 at `qabs`.
static int mla_q_stage(const qcau_mla_dims* d, const void* q_lora, const void* wq_b,
                       const void* wq_b_scale, const void* wkv_b_bf16, const int32_t* positions,
                       const float* freqs, void* qabs, uint8_t* ws, const MlaWs& w,
                       cudaStream_t st) {
  const int64_t B = d->batch, H = d->n_heads;
  const int64_t dq = d->d_nope + d->d_rope;
  const int64_t dabs = d->kv_lora + d->d_rope;
  const int a_e8 = d->act_round_scale ? 1 : 0;
  const int w_e8 = d->w_scale_dtype == QCAU_SCALE_E8M0;
  // q = wq_b(act_quant(q_lora))
  QCAU_CHECK_CUDA(launch_act_quant(q_lora, ws + w.xq, ws + w.sq, B, d->dc, 128,
                                   d->act_round_scale, a_e8, 0, st));
  QCAU_CHECK_CUDA(launch_fp8_gemm(ws + w.xq, ws + w.sq, wq_b, wq_b_scale, ws + w.q, B, H * dq,
                                  d->dc, a_e8, w_e8, 0, st));
  // RoPE on q_rope (last 64 of each head) at each sequence's position, in
  // place and into the rope slot of q_abs (q_abs[:, :, kv_lora:]): done by
  // the absorb's epilogue threads for the 64-dim rope of the 512-wide
  // latent, by its own launch otherwise
  uint8_t* qa = reinterpret_cast<uint8_t*>(qabs);
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  const bool fused_rope = d->d_rope == 64 && d->kv_lora % 256 == 0 && d->d_nope == 128 &&
                          dq % 8 == 0 && dabs % 8 == 0 && al16(ws + w.q) && al16(qa) &&
                          al16(freqs);
  if (!fused_rope)
    QCAU_CHECK_CUDA(launch_rope_pairs(ws + w.q + d->d_nope * 2, dq, qa + d->kv_lora * 2, dabs,
                                      freqs, positions, B, 1, H, (int)d->d_rope, 0, 0, st));
  // q_abs[:, :, :512] = q_nope . W_UK ;  q_abs[:, :, 512:] = q_rope
  BmmArgs m{};
  if (fused_rope) {
    m.rope_x = ws + w.q + d->d_nope * 2;
    m.rope_x_stride = dq;
    m.rope_copy = qa + d->kv_lora * 2;
    m.rope_copy_stride = dabs;
    m.rope_freqs = freqs;
    m.rope_pos = positions;
  }
  m.a = ws + w.q;
  m.a_bstride = dq;
  m.a_rstride = H * dq;
  m.b = wkv_b_bf16;
  m.b_bstride = (d->d_nope + d->d_v) * d->kv_lora;
  m.b_rstride = d->kv_lora;
  m.b_kmajor = 0;
  m.c = qa;
  m.c_bstride = dabs;
  m.c_rstride = H * dabs;
  m.batch = H;
  m.m = B;
  m.n = d->kv_lora;
  m.k = d->d_nope;
  QCAU_CHECK_CUDA(launch_bf16_bmm(m, st));
  return QCAU_OK;
}

// Output side of the layer: o_lat [B, H, kv_lora] bf16 -> y.
static int mla_out_stage(const qcau_mla_dims* d, const void* olat, const void* wkv_b_bf16,
                         const void* wo, const void* wo_scale, void* y, uint8_t* ws,
                         const MlaWs& w, cudaStream_t st) {
  const int64_t B = d->batch, H = d->n_heads;
  const int a_e8 = d->act_round_scale ? 1 : 0;
  const int w_e8 = d->w_scale_dtype == QCAU_SCALE_E8M0;
  // o_v = o_lat . W_UV^T
  BmmArgs m{};
  m.a = olat;
  m.a_bstride = d->kv_lora;
  m.a_rstride = H * d->kv_lora;
  m.b = reinterpret_cast<const uint8_t*>(wkv_b_bf16) + d->d_nope * d->kv_lora * 2;
  m.b_bstride = (d->d_nope + d->d_v) * d->kv_lora;
  m.b_rstride = d->kv_lora;
  m.b_kmajor = 1;
  m.c = ws + w.ov;
  m.c_bstride = d->d_v;
  m.c_rstride = H * d->d_v;
  m.batch = H;
  m.m = B;
  m.n = d->d_v;
  m.k = d->kv_lora;
  // act_quant(o_v) in 1 x 128 blocks (one head's d_v values a block) comes
  // out of the same epilogue: FP8 codes at x_o, scales at s_o
  const bool fused_quant = d->d_v == 128;
  if (fused_quant) {
    m.q_codes = ws + w.xo;
    m.q_scales = ws + w.so;
    m.q_round_scale = d->act_round_scale;
    m.q_scale_e8m0 = a_e8;
  }
  QCAU_CHECK_CUDA(launch_bf16_bmm(m, st));
  // y = wo(act_quant(o_v))   (row-parallel partial; the caller all-reduces)
  if (!fused_quant)
    QCAU_CHECK_CUDA(launch_act_quant(ws + w.ov, ws + w.xo, ws + w.so, B, H * d->d_v, 128,
                                     d->act_round_scale, a_e8, 0, st));
  QCAU_CHECK_CUDA(launch_fp8_gemm(ws + w.xo, ws + w.so, wo, wo_scale, y, B, d->dim, H * d->d_v,
                                  a_e8, w_e8, d->out_dtype == QCAU_OUT_F32, st));
  return QCAU_OK;
}

int qcau_mla_decode(const qcau_mla_dims* d, const void* q_lora, const void* wq_b,
                    const void* wq_b_scale, const void* wkv_b_bf16, const void* wo,
                    const void* wo_scale, const void* cache, const int32_t* block_table,
                    const int32_t* seqlens, const int32_t* positions, const float* freqs, void* y,
                    void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_mla_dims(d, "mla_decode");
  if (rc) return rc;
  QCAU_CHECK_ARG(q_lora && wq_b && wq_b_scale && wkv_b_bf16 && wo && wo_scale && cache &&
                     block_table && seqlens && positions && freqs && y,
                 "mla_decode: NULL pointer");
  QCAU_CHECK_ARG(d->max_seqlen >= 0 && d->max_seqlen <= d->max_pages * d->page_size,
                 "mla_decode: max_seqlen exceeds the block table");
  const MlaWs w = mla_ws(d);
  if (workspace_bytes < w.total || !workspace)
    return fail(QCAU_ERR_WORKSPACE, "mla_decode: workspace too small (need " +
                                        std::to_string(w.total) + " bytes)");
  if (d->batch == 0) return QCAU_OK;
  cudaStream_t st = to_stream(stream);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const int64_t dabs = d->kv_lora + d->d_rope;
  rc = mla_q_stage(d, q_lora, wq_b, wq_b_scale, wkv_b_bf16, positions, freqs, ws + w.qabs, ws, w,
                   st);
  if (rc) return rc;
  // o_lat = attention over the paged latent cache (V = first 512 of each row)
  {
    AttnArgs a{};
    a.q = ws + w.qabs;
    a.q_row_stride = dabs;
    a.kv = cache;
    a.block_table = block_table;
    a.seqlens = seqlens;
    a.sink = nullptr;
    a.o = ws + w.olat;
    a.b = d->batch; a.s = 1; a.h = d->n_heads; a.d_qk = dabs; a.d_v = d->kv_lora; a.d_kv = dabs;
    a.page_size = d->page_size;
    a.max_pages = d->max_pages;
    a.num_pages = d->num_pages;
    a.max_len = d->max_seqlen;
    a.scale = d->softmax_scale;
    rc = run_decode_attn(a, ws + w.attn, st);
    if (rc) return rc;
  }
  return mla_out_stage(d, ws + w.olat, wkv_b_bf16, wo, wo_scale, y, ws, w, st);
}

int qcau_mla_decode_q(const qcau_mla_dims* d, const void* q_lora, const void* wq_b,
                      const void* wq_b_scale, const void* wkv_b_bf16, const int32_t* positions,
                      const float* freqs, void* q_abs, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc = check_mla_dims(d, "mla_decode_q");
  if (rc) return rc;
  QCAU_CHECK_ARG(q_lora && wq_b && wq_b_scale && wkv_b_bf16 && positions && freqs && q_abs,
                 "mla_decode_q: NULL pointer");
  const MlaWs w = mla_ws(d);
  if (workspace_bytes < w.total || !workspace)
    return fail(QCAU_ERR_WORKSPACE, "mla_decode_q: workspace too small (need " +
                                        std::to_string(w.total) + " bytes)");
  if (d->batch == 0) return QCAU_OK;
  return mla_q_stage(d, q_lora, wq_b, wq_b_scale, wkv_b_bf16, positions, freqs, q_abs,
                     reinterpret_cast<uint8_t*>(workspace), w, to_stream(stream));
}

int qcau_mla_decode_out(const qcau_mla_dims* d, const void* o_lat, const void* wkv_b_bf16,
                        const void* wo, const void* wo_scale, void* y, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_mla_dims(d, "mla_decode_out");
  if (rc) return rc;
  QCAU_CHECK_ARG(o_lat && wkv_b_bf16 && wo && wo_scale && y, "mla_decode_out: NULL pointer");
  const MlaWs w = mla_ws(d);
  if (workspace_bytes < w.total || !workspace)
    return fail(QCAU_ERR_WORKSPACE, "mla_decode_out: workspace too small (need " +
                                        std::to_string(w.total) + " bytes)");
  if (d->batch == 0) return QCAU_OK;
  return mla_out_stage(d, o_lat, wkv_b_bf16, wo, wo_scale, y,
                       reinterpret_cast<uint8_t*>(workspace), w, to_stream(stream));
}

int qcau_decode_attn_paged_cp(const void* q_all, const void* cache, const int32_t* block_table,
                              const int32_t* seqlens, void* part_o, float* part_ml, int64_t b,
                              int64_t h, int64_t n_ranks, int64_t rank, int64_t d_qk, int64_t d_v,
                              int64_t d_kv, int64_t page_size, int64_t max_pages,
                              int64_t num_pages, int64_t max_seqlen, float softmax_scale,
                              int32_t part_f16, void* stream) {
  QCAU_CHECK_ARG(q_all && cache && block_table && seqlens && part_o && part_ml,
                 "decode_attn_paged_cp: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "decode_attn_paged_cp: bad shape");
  QCAU_CHECK_ARG(n_ranks >= 1 && rank >= 0 && rank < n_ranks && h % n_ranks == 0,
                 "decode_attn_paged_cp: rank out of range or heads not divisible by ranks");
  QCAU_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= max_pages * page_size,
                 "decode_attn_paged_cp: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "decode_attn_paged_cp");
  if (rc) return rc;
  AttnArgs a{};
  a.q = q_all;
  a.q_row_stride = d_qk;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.b = b; a.s = 1; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  a.splits = 1;
  a.split_base = (int)rank;
  a.splits_total = (int)n_ranks;
  a.q_hblock = h / n_ranks;
  a.part_hblock = h / n_ranks;
  a.part_o = reinterpret_cast<float*>(part_o);
  a.part_ml = part_ml;
  a.part_f16 = part_f16 ? 1 : 0;
  if (!decode_attn_sm100_supported(a))
    return fail(QCAU_ERR_UNSUPPORTED,
                "decode_attn_paged_cp: needs the sm_100a pair kernel (d_qk 576, d_v 512, page 64, "
                "h a multiple of 128, h / n_ranks a multiple of 64 or 8, 16 or 32)");
  if (b == 0) return QCAU_OK;
  QCAU_CHECK_CUDA(launch_decode_attn_sm100(a, to_stream(stream)));
  return QCAU_OK;
}

int qcau_decode_attn_paged_cp_p2p(const void* q_all, const void* cache,
                                  const int32_t* block_table, const int32_t* seqlens,
                                  void* const* dst_o, float* const* dst_ml,
                                  uint32_t* const* dst_flag, uint32_t epoch,
                                  uint32_t* done_counter, int64_t b, int64_t h, int64_t n_ranks,
                                  int64_t rank, int64_t d_qk, int64_t d_v, int64_t d_kv,
                                  int64_t page_size, int64_t max_pages, int64_t num_pages,
                                  int64_t max_seqlen, float softmax_scale, int32_t part_f16,
                                  void* stream) {
  QCAU_CHECK_ARG(q_all && cache && block_table && seqlens && dst_o && dst_ml && dst_flag &&
                     done_counter,
                 "decode_attn_paged_cp_p2p: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h > 0 && page_size > 0 && max_pages > 0 && num_pages > 0,
                 "decode_attn_paged_cp_p2p: bad shape");
  QCAU_CHECK_ARG(n_ranks >= 1 && n_ranks <= 16 && rank >= 0 && rank < n_ranks && h % n_ranks == 0,
                 "decode_attn_paged_cp_p2p: 1..16 ranks, rank in range, heads divisible by ranks");
  for (int64_t j = 0; j < n_ranks; j++)
    QCAU_CHECK_ARG(dst_o[j] && dst_ml[j] && dst_flag[j],
                   "decode_attn_paged_cp_p2p: NULL destination pointer");
  QCAU_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= max_pages * page_size,
                 "decode_attn_paged_cp_p2p: max_seqlen exceeds the block table");
  int rc = check_attn_widths(d_qk, d_v, d_kv, "decode_attn_paged_cp_p2p");
  if (rc) return rc;
  AttnArgs a{};
  a.q = q_all;
  a.q_row_stride = d_qk;
  a.kv = cache;
  a.block_table = block_table;
  a.seqlens = seqlens;
  a.b = b; a.s = 1; a.h = h; a.d_qk = d_qk; a.d_v = d_v; a.d_kv = d_kv;
  a.page_size = page_size;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.max_len = max_seqlen;
  a.scale = softmax_scale;
  a.splits = 1;
  a.split_base = (int)rank;
  a.splits_total = (int)n_ranks;
  a.q_hblock = h / n_ranks;
  a.part_hblock = h / n_ranks;
  a.peer = 1;
  for (int64_t j = 0; j < n_ranks; j++) {
    a.peer_o[j] = dst_o[j];
    a.peer_ml[j] = dst_ml[j];
    a.peer_flag[j] = dst_flag[j];
  }
  a.done_counter = done_counter;
  a.epoch = epoch;
  a.part_f16 = part_f16 ? 1 : 0;
  if (!decode_attn_sm100_supported(a))
    return fail(QCAU_ERR_UNSUPPORTED,
                "decode_attn_paged_cp_p2p: needs the sm_100a pair kernel (d_qk 576, d_v 512, "
                "page 64, h a multiple of 128, h / n_ranks a multiple of 64 or 8, 16 or 32)");
  if (b == 0) return QCAU_OK;
  QCAU_CHECK_CUDA(launch_decode_attn_sm100(a, to_stream(stream)));
  return QCAU_OK;
}

int qcau_wait_flags(const uint32_t* flags, int64_t n, uint32_t epoch, void* stream) {
  QCAU_CHECK_ARG(flags != nullptr && n >= 0 && n <= 1024, "wait_flags: bad argument");
  QCAU_CHECK_CUDA(launch_wait_flags(flags, (int)n, epoch, to_stream(stream)));
  return QCAU_OK;
}

size_t qcau_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int qcau_ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
  QCAU_CHECK_ARG(ptr != nullptr && handle_out != nullptr && bytes > 0, "ipc_alloc: bad argument");
  void* p = nullptr;
  QCAU_CHECK_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail_cuda(e, "ipc_alloc");
  }
  *ptr = p;
  return QCAU_OK;
}

int qcau_ipc_open(const void* handle, void** ptr) {
  QCAU_CHECK_ARG(handle != nullptr && ptr != nullptr, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  QCAU_CHECK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return QCAU_OK;
}

int qcau_ipc_close(void* ptr) {
  QCAU_CHECK_ARG(ptr != nullptr, "ipc_close: NULL pointer");
  QCAU_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
  return QCAU_OK;
}

int qcau_ipc_free(void* ptr) {
  QCAU_CHECK_ARG(ptr != nullptr, "ipc_free: NULL pointer");
  QCAU_CHECK_CUDA(cudaFree(ptr));
  return QCAU_OK;
}

int qcau_attn_combine_ranks(const void* part_o, const float* part_ml, const float* attn_sink,
                            void* o, int64_t b, int64_t h_local, int64_t n_ranks, int64_t d_v,
                            int32_t part_f16, void* stream) {
  QCAU_CHECK_ARG(part_o && part_ml && o, "attn_combine_ranks: NULL pointer");
  QCAU_CHECK_ARG(b >= 0 && h_local > 0 && n_ranks >= 1 && d_v > 0 && d_v % 128 == 0,
                 "attn_combine_ranks: bad shape");
  AttnArgs a{};
  a.part_o = const_cast<float*>(reinterpret_cast<const float*>(part_o));
  a.part_f16 = part_f16 ? 1 : 0;
  a.part_ml = const_cast<float*>(part_ml);
  a.sink = attn_sink;
  a.o = o;
  a.b = b; a.s = 1; a.h = h_local; a.d_v = d_v;
  a.splits = (int)n_ranks;
  a.part_split_major = 1;
  QCAU_CHECK_CUDA(launch_attn_combine(a, to_stream(stream)));
  return QCAU_OK;
}

}  // extern "C"
