/*
 * qcau_oracle.c -- CPU restatement of the reference QCAU path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA product
 * path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * load it.  The product library never links or calls it.
 *
 * Every function names the reference lines it restates (paths relative to the
 * reference project root).  Parity of this restatement is pinned against the
 * reference's own golden vectors (QCAU/QCAU_inference/framework/test_vectors)
 * and against the reference's PyTorch path run in-process on synthetic
 * inputs; see tests/test_oracle_pins.py and tests/golden/make_golden.py.
 *
 * Number formats
 *   bf16  : uint16_t bit pattern, round-to-nearest-even from fp32
 *   e4m3  : uint8_t  bit pattern (float8_e4m3fn: bias 7, max 448, no inf)
 *   e8m0  : uint8_t  bit pattern, value 2^(b-127)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

/* ------------------------------------------------------------------ */
/* scalar formats                                                      */
/* ------------------------------------------------------------------ */

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float bf16_round(float f) { return orc_bf16_to_f32(orc_f32_to_bf16(f)); }

float orc_e4m3_to_f32(uint8_t b) {
    int sign = b >> 7;
    int e = (b >> 3) & 0xf;
    int m = b & 7;
    float v;
    if (e == 0xf && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
    return sign ? -v : v;
}

/* fp32 -> e4m3fn, round to nearest even, saturating to +-448 (the
 * reference clamps to +-448 before the cast, kernel.py:93-96). */
uint8_t orc_f32_to_e4m3(float x) {
    if (isnan(x)) return 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    float a = fabsf(x);
    if (a >= 448.0f) return sign | 0x7e;
    if (a < ldexpf(1.0f, -6)) {
        /* subnormal grid: multiples of 2^-9; scaling by 2^9 is exact */
        float q = nearbyintf(ldexpf(a, 9));
        int qi = (int)q;            /* 0..8; 8 == smallest normal 2^-6 */
        if (qi >= 8) return sign | (1 << 3);
        return sign | (uint8_t)qi;
    }
    int e;
    float fr = frexpf(a, &e);       /* a = fr * 2^e, fr in [0.5,1) */
    /* a = (1+m/8) * 2^(e-1) with mantissa fr*16-8 in [0,8) */
    float mq = nearbyintf(fr * 16.0f) - 8.0f;
    int E = e - 1;
    int mi = (int)mq;
    if (mi == 8) { mi = 0; E += 1; }
    int field = E + 7;
    if (field > 15 || (field == 15 && mi == 7)) return sign | 0x7e;
    return sign | (uint8_t)((field << 3) | mi);
}

float orc_e8m0_to_f32(uint8_t b) {
    if (b == 0xff) return NAN;
    return ldexpf(1.0f, (int)b - 127);
}

uint8_t orc_f32_pow2_to_e8m0(float s) {
    uint32_t u;
    memcpy(&u, &s, 4);
    return (uint8_t)((u >> 23) & 0xff);
}

/* ------------------------------------------------------------------ */
/* act_quant: Deepseek_origin/inference/kernel.py:40-125               */
/*   amax = max(|x| over 1 x block, 1e-4)                 (:77-79)     */
/*   s    = amax / 448             or, with round_scale,              */
/*          2^ceil(log2(amax / 448)) by exponent bits     (:22-37,:81) */
/*   y    = e4m3(clamp(x / s, -448, 448))                 (:93-96)     */
/*   inplace: y = bf16(f32(e4m3(clamp(x/s))) * s)         (:84-91)     */
/* ------------------------------------------------------------------ */

static float act_scale(float amax, int round_scale) {
    if (amax < 1e-4f) amax = 1e-4f;
    /* amax / 448 correctly rounded, as kernel_fallback.py:27-28 computes it
     * (kernel.py:83 multiplies by fl(1/448) instead, which differs in the
     * last bit for about half of all blocks; the fallback is the reference
     * path that runs and is pinned here).  The UE8M0 rounding takes the
     * exponent bits exactly as kernel.py:22-37 does. */
    float t = amax / 448.0f;
    if (!round_scale) return t;
    uint32_t bits;
    memcpy(&bits, &t, 4);
    int ex = (int)((bits >> 23) & 0xff);
    uint32_t man = bits & 0x7fffffu;
    int e = ex - 127 + (man != 0 ? 1 : 0);
    uint32_t ob = (uint32_t)(e + 127) << 23;
    float s;
    memcpy(&s, &ob, 4);
    return s;
}

void orc_act_quant(const uint16_t* x, int64_t m, int64_t n, int block,
                   int round_scale, uint8_t* y, float* s) {
    int64_t nb = n / block;
    for (int64_t r = 0; r < m; r++) {
        for (int64_t b = 0; b < nb; b++) {
            const uint16_t* xb = x + r * n + b * block;
            float amax = 0.0f;
            for (int j = 0; j < block; j++) {
                float v = fabsf(orc_bf16_to_f32(xb[j]));
                if (v > amax) amax = v;
            }
            float sc = act_scale(amax, round_scale);
            s[r * nb + b] = sc;
            for (int j = 0; j < block; j++) {
                float v = orc_bf16_to_f32(xb[j]) / sc;
                if (v > 448.0f) v = 448.0f;
                if (v < -448.0f) v = -448.0f;
                y[r * n + b * block + j] = orc_f32_to_e4m3(v);
            }
        }
    }
}

void orc_act_quant_inplace(uint16_t* x, int64_t m, int64_t n, int block,
                           int round_scale) {
    int64_t nb = n / block;
    for (int64_t r = 0; r < m; r++) {
        for (int64_t b = 0; b < nb; b++) {
            uint16_t* xb = x + r * n + b * block;
            float amax = 0.0f;
            for (int j = 0; j < block; j++) {
                float v = fabsf(orc_bf16_to_f32(xb[j]));
                if (v > amax) amax = v;
            }
            float sc = act_scale(amax, round_scale);
            for (int j = 0; j < block; j++) {
                float v = orc_bf16_to_f32(xb[j]) / sc;
                if (v > 448.0f) v = 448.0f;
                if (v < -448.0f) v = -448.0f;
                float dq = orc_e4m3_to_f32(orc_f32_to_e4m3(v)) * sc;
                xb[j] = orc_f32_to_bf16(dq);
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* fp8_gemm: Deepseek_origin/inference/kernel.py:203-273 and           */
/* qcau_c/src/qcau.cpp:30-90.  Two-level accumulation: each 128-wide   */
/* K block is summed in fp32, then promoted with sa[m,kb]*sb[n/128,kb] */
/* into a second fp32 accumulator (kernel.py:242-250).                 */
/* ------------------------------------------------------------------ */

void orc_fp8_gemm(const uint8_t* a, const float* sa, const uint8_t* b,
                  const float* sb, int64_t m, int64_t n, int64_t k,
                  float* c) {
    int64_t kb = (k + 127) / 128;
    #pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; j++) {
        float* bf = (float*)malloc(sizeof(float) * (size_t)k);
        float* af = (float*)malloc(sizeof(float) * (size_t)k);
        for (int64_t t = 0; t < k; t++) bf[t] = orc_e4m3_to_f32(b[j * k + t]);
        for (int64_t i = 0; i < m; i++) {
            for (int64_t t = 0; t < k; t++) af[t] = orc_e4m3_to_f32(a[i * k + t]);
            float acc = 0.0f;
            for (int64_t q = 0; q < kb; q++) {
                float part = 0.0f;
                int64_t t1 = (q + 1) * 128 < k ? (q + 1) * 128 : k;
                for (int64_t t = q * 128; t < t1; t++) part += af[t] * bf[t];
                float scale = sa[i * kb + q] * sb[(j / 128) * kb + q];
                acc += part * scale;
            }
            c[i * n + j] = acc;
        }
        free(bf);
        free(af);
    }
}

/* ------------------------------------------------------------------ */
/* Per-head RMSNorm in bf16 arithmetic: Deepseek_origin/inference/     */
/* model.py:498 `q *= rsqrt(q.square().mean(-1) + eps)` on a bf16      */
/* tensor, i.e. QCAU/QCAU_inference/inference/QCAU.py:16-27 with the   */
/* optional per-head gamma.  Each elementwise op rounds to bf16; the   */
/* mean reduction accumulates in fp32.                                 */
/* ------------------------------------------------------------------ */

void orc_head_rms_norm(uint16_t* x, int64_t rows, int64_t d,
                       const uint16_t* gamma, int64_t n_heads, float eps) {
    for (int64_t r = 0; r < rows; r++) {
        uint16_t* xr = x + r * d;
        float acc = 0.0f;
        for (int64_t j = 0; j < d; j++) {
            float v = orc_bf16_to_f32(xr[j]);
            acc += bf16_round(v * v);
        }
        float mean = bf16_round(acc / (float)d);
        float rs = bf16_round(1.0f / sqrtf(bf16_round(mean + eps)));
        const uint16_t* g = gamma ? gamma + (r % n_heads) * d : NULL;
        for (int64_t j = 0; j < d; j++) {
            float y = bf16_round(orc_bf16_to_f32(xr[j]) * rs);
            if (g) y = bf16_round(y * orc_bf16_to_f32(g[j]));
            xr[j] = orc_f32_to_bf16(y);
        }
    }
}

/* ------------------------------------------------------------------ */
/* RoPE on the last `rope_dim` values of each row, interleaved pairs   */
/* (2i, 2i+1): Deepseek_origin/inference/model.py:231-243,             */
/* QCAU/QCAU_inference/inference/QCAU.py:30-68.  fp32 complex multiply,*/
/* bf16 store.  freqs is [positions, rope_dim/2, 2] fp32 (re, im).     */
/* rows are [B, S, H] flattened; the position of row r is              */
/* pos0 + (r / n_heads) % seqlen.                                      */
/* ------------------------------------------------------------------ */

void orc_rope(uint16_t* x, int64_t rows, int64_t row_stride, int64_t d,
              int64_t rope_dim, const float* freqs, int64_t n_heads,
              int64_t seqlen, int64_t pos0, int inverse) {
    int64_t np = rope_dim / 2;
    for (int64_t r = 0; r < rows; r++) {
        int64_t pos = pos0 + (r / n_heads) % seqlen;
        uint16_t* t = x + r * row_stride + (d - rope_dim);
        const float* f = freqs + pos * np * 2;
        for (int64_t i = 0; i < np; i++) {
            float a = orc_bf16_to_f32(t[2 * i]);
            float b = orc_bf16_to_f32(t[2 * i + 1]);
            float c = f[2 * i];
            float s = inverse ? -f[2 * i + 1] : f[2 * i + 1];
            float re = a * c - b * s;
            float im = a * s + b * c;
            t[2 * i] = orc_f32_to_bf16(re);
            t[2 * i + 1] = orc_f32_to_bf16(im);
        }
    }
}

/* ------------------------------------------------------------------ */
/* KV build: Deepseek_origin/inference/model.py:502-506, in place on   */
/* rows [rows, d] bf16:                                                */
/*   RMSNorm of values [0, norm_dim) (model.py:182-195): fp32 squares, */
/*   var = mean, x * (1 / sqrt(var + eps)) (torch's CPU rsqrt), times  */
/*   the fp32 weight, rounded to bf16 once                             */
/*   RoPE of the last rope_dim values at positions[r] (:231-243)       */
/*   act_quant(kv[..., :quant_dims], 64, fmt, inplace=True) (:505)     */
/* ------------------------------------------------------------------ */
void orc_kv_build(uint16_t* x, int64_t rows, int64_t d, const float* w,
                  int64_t norm_dim, float eps, const float* freqs,
                  const int32_t* positions, int64_t rope_dim,
                  int64_t quant_dims, int round_scale) {
    for (int64_t r = 0; r < rows; r++) {
        uint16_t* xr = x + r * d;
        if (norm_dim > 0) {
            float acc = 0.0f;
            for (int64_t j = 0; j < norm_dim; j++) {
                float v = orc_bf16_to_f32(xr[j]);
                acc += v * v;
            }
            float rs = 1.0f / sqrtf(acc / (float)norm_dim + eps);
            for (int64_t j = 0; j < norm_dim; j++) {
                float v = orc_bf16_to_f32(xr[j]) * rs;
                xr[j] = orc_f32_to_bf16((w ? w[j] : 1.0f) * v);
            }
        }
        if (rope_dim > 0)
            orc_rope(xr, 1, d, d, rope_dim, freqs, 1, 1, positions[r], 0);
        if (quant_dims > 0) orc_act_quant_inplace(xr, 1, quant_dims, 64, round_scale);
    }
}

/* ------------------------------------------------------------------ */
/* Attention core: Deepseek_origin/inference/kernel.py:276-352 with    */
/* the guards of QCAU/QCAU_inference/inference/QCAU.py:176-242 and the */
/* bf16 rounding of P before P.V (kernel.py:340, check/QCAU.py:263).   */
/*   tile of 64 indices; index outside [0, n_kv) -> score -inf, row 0  */
/*   m_new = max(m, tile max) only if the tile has a valid index       */
/*   l = l*alpha + sum(p);  acc = acc*alpha + sum(bf16(p) * v)         */
/*   l += exp(sink - m) once at the end (kernel.py:345-346)            */
/* K rows are kv[..., :d_qk]; V rows are kv[..., :d_v] (V4: equal;     */
/* absorbed MLA: d_qk = 576, d_v = 512).                               */
/* row_of(b, idx) gives the kv row pointer (dense [B,N,D] or paged).   */
/* ------------------------------------------------------------------ */

typedef const uint16_t* (*row_fn)(const void* ctx, int64_t b, int64_t idx);

struct dense_ctx { const uint16_t* kv; int64_t n; int64_t d; };
static const uint16_t* dense_row(const void* c, int64_t b, int64_t idx) {
    const struct dense_ctx* d = (const struct dense_ctx*)c;
    return d->kv + (b * d->n + idx) * d->d;
}

struct paged_ctx { const uint16_t* cache; const int32_t* table; int64_t max_pages;
                   int64_t page; int64_t d; };
static const uint16_t* paged_row(const void* c, int64_t b, int64_t idx) {
    const struct paged_ctx* p = (const struct paged_ctx*)c;
    int64_t blk = p->table[b * p->max_pages + idx / p->page];
    return p->cache + (blk * p->page + idx % p->page) * p->d;
}

static void attn_one(const uint16_t* q, int64_t h_count, int64_t d_qk, int64_t d_v,
                     const void* ctx, row_fn row, int64_t b, const int32_t* idx,
                     int64_t topk, int64_t n_kv, const float* sink, float scale,
                     float* out /* [h_count, d_v] */, float* lse /* [h_count] or NULL */) {
    const int64_t T = 64;
    float* qf = (float*)malloc(sizeof(float) * (size_t)(h_count * d_qk));
    float* acc = (float*)calloc((size_t)(h_count * d_v), sizeof(float));
    float* mx = (float*)malloc(sizeof(float) * (size_t)h_count);
    float* l = (float*)calloc((size_t)h_count, sizeof(float));
    float sc[64];
    float* rows = (float*)malloc(sizeof(float) * (size_t)(T * d_qk));
    int valid[64];
    for (int64_t i = 0; i < h_count * d_qk; i++) qf[i] = orc_bf16_to_f32(q[i]);
    for (int64_t h = 0; h < h_count; h++) mx[h] = -INFINITY;
    for (int64_t t0 = 0; t0 < topk; t0 += T) {
        int any = 0;
        for (int64_t i = 0; i < T; i++) {
            int64_t j = t0 + i;
            int64_t id = j < topk ? idx[j] : -1;
            valid[i] = (id >= 0 && id < n_kv);
            any |= valid[i];
            if (valid[i]) {
                const uint16_t* r = row(ctx, b, id);
                for (int64_t c = 0; c < d_qk; c++) rows[i * d_qk + c] = orc_bf16_to_f32(r[c]);
            } else {
                for (int64_t c = 0; c < d_qk; c++) rows[i * d_qk + c] = 0.0f;
            }
        }
        if (!any) continue;
        for (int64_t h = 0; h < h_count; h++) {
            float tmax = -INFINITY;
            for (int64_t i = 0; i < T; i++) {
                if (!valid[i]) { sc[i] = -INFINITY; continue; }
                float dot = 0.0f;
                for (int64_t c = 0; c < d_qk; c++) dot += qf[h * d_qk + c] * rows[i * d_qk + c];
                sc[i] = dot * scale;
                if (sc[i] > tmax) tmax = sc[i];
            }
            float mnew = mx[h] > tmax ? mx[h] : tmax;
            float alpha = expf(mx[h] - mnew);
            float psum = 0.0f;
            float* a = acc + h * d_v;
            for (int64_t c = 0; c < d_v; c++) a[c] *= alpha;
            for (int64_t i = 0; i < T; i++) {
                if (!valid[i]) continue;
                float p = expf(sc[i] - mnew);
                psum += p;
                float pb = bf16_round(p);
                for (int64_t c = 0; c < d_v; c++) a[c] += pb * rows[i * d_qk + c];
            }
            l[h] = l[h] * alpha + psum;
            mx[h] = mnew;
        }
    }
    for (int64_t h = 0; h < h_count; h++) {
        float sk = sink ? sink[h] : -INFINITY;
        float term;
        if (isfinite(mx[h])) term = expf(sk - mx[h]);
        else term = isfinite(sk) ? 1.0f : 0.0f;
        float den = l[h] + term;
        if (den < FLT_MIN) den = FLT_MIN;
        for (int64_t c = 0; c < d_v; c++) out[h * d_v + c] = acc[h * d_v + c] / den;
        if (lse) lse[h] = isfinite(mx[h]) ? mx[h] + logf(den) : -INFINITY;
    }
    free(qf); free(acc); free(mx); free(l); free(rows);
}

/* q [B,S,H,d_qk] bf16, kv [B,N,d_kv] bf16 (d_kv >= d_qk), idx [B,S,K]
 * out [B,S,H,d_v] fp32 (caller rounds to bf16 as the kernel does). */
void orc_sparse_attn(const uint16_t* q, const uint16_t* kv, const float* sink,
                     const int32_t* idx, int64_t bsz, int64_t s, int64_t h,
                     int64_t d_qk, int64_t d_v, int64_t d_kv, int64_t n_kv,
                     int64_t topk, float scale, float* out) {
    struct dense_ctx ctx = { kv, n_kv, d_kv };
    #pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < bsz; b++)
        for (int64_t t = 0; t < s; t++)
            attn_one(q + ((b * s + t) * h) * d_qk, h, d_qk, d_v, &ctx, dense_row, b,
                     idx + (b * s + t) * topk, topk, n_kv, sink, scale,
                     out + ((b * s + t) * h) * d_v, NULL);
}

/* Dense decode over a paged cache: every sequence attends to all of its
 * first seqlens[b] tokens (one query token per sequence).  This is the
 * same core with idx = 0..seqlen-1 mapped through the block table.
 * cache [num_pages, page, d_kv] bf16, table [B, max_pages] int32. */
void orc_paged_decode_attn(const uint16_t* q, const uint16_t* cache,
                           const int32_t* table, const int32_t* seqlens,
                           const float* sink, int64_t bsz, int64_t h,
                           int64_t d_qk, int64_t d_v, int64_t d_kv,
                           int64_t page, int64_t max_pages, float scale,
                           float* out, float* lse) {
    struct paged_ctx ctx = { cache, table, max_pages, page, d_kv };
    #pragma omp parallel for schedule(dynamic)
    for (int64_t b = 0; b < bsz; b++) {
        int64_t n = seqlens[b];
        int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
        for (int64_t i = 0; i < n; i++) idx[i] = (int32_t)i;
        attn_one(q + b * h * d_qk, h, d_qk, d_v, &ctx, paged_row, b, idx, n, n, sink,
                 scale, out + b * h * d_v, lse ? lse + b * h : NULL);
        free(idx);
    }
}

/* ------------------------------------------------------------------ */
/* Absorbed-MLA extras.  The reference has no code for these (its V4  */
/* attention has no wkv_b); they restate the standard MLA absorption   */
/* with wkv_b [H*(d_nope+d_v), kv_lora] dequantised to bf16:           */
/*   absorb: q_lat[b,h,j] = sum_c q_nope[b,h,c] * wkv_b[h*(dn+dv)+c, j]*/
/*   v-up  : o_v[b,h,d]   = sum_c o_lat[b,h,c] * wkv_b[h*(dn+dv)+dn+d, c]*/
/* fp32 accumulation, bf16 result.                                     */
/* ------------------------------------------------------------------ */

void orc_mla_absorb(const uint16_t* q, int64_t q_row_stride, const uint16_t* wkv,
                    int64_t bsz, int64_t h, int64_t d_nope, int64_t d_v,
                    int64_t kv_lora, uint16_t* q_lat, int64_t out_row_stride) {
    #pragma omp parallel for collapse(2)
    for (int64_t b = 0; b < bsz; b++)
        for (int64_t hh = 0; hh < h; hh++) {
            const uint16_t* qn = q + (b * h + hh) * q_row_stride;
            const uint16_t* w = wkv + hh * (d_nope + d_v) * kv_lora;
            for (int64_t j = 0; j < kv_lora; j++) {
                float acc = 0.0f;
                for (int64_t c = 0; c < d_nope; c++)
                    acc += orc_bf16_to_f32(qn[c]) * orc_bf16_to_f32(w[c * kv_lora + j]);
                q_lat[(b * h + hh) * out_row_stride + j] = orc_f32_to_bf16(acc);
            }
        }
}

void orc_mla_vup(const uint16_t* o_lat, const uint16_t* wkv, int64_t bsz, int64_t h,
                 int64_t d_nope, int64_t d_v, int64_t kv_lora, uint16_t* o_v) {
    #pragma omp parallel for collapse(2)
    for (int64_t b = 0; b < bsz; b++)
        for (int64_t hh = 0; hh < h; hh++) {
            const uint16_t* o = o_lat + (b * h + hh) * kv_lora;
            const uint16_t* w = wkv + (hh * (d_nope + d_v) + d_nope) * kv_lora;
            for (int64_t d = 0; d < d_v; d++) {
                float acc = 0.0f;
                for (int64_t c = 0; c < kv_lora; c++)
                    acc += orc_bf16_to_f32(o[c]) * orc_bf16_to_f32(w[d * kv_lora + c]);
                o_v[(b * h + hh) * d_v + d] = orc_f32_to_bf16(acc);
            }
        }
}

/* Grouped low-rank projection wo_a: Deepseek_origin/inference/model.py:  */
/* 537-541, einsum("bsgd,grd->bsgr", o, wo_a) in bf16 (fp32 sums, bf16   */
/* result): o [rows, groups, gd], w [groups, rank, gd] -> h [rows, groups, */
/* rank].                                                                 */
void orc_grouped_proj(const uint16_t* o, const uint16_t* w, int64_t rows, int64_t groups,
                      int64_t gd, int64_t rank, uint16_t* h) {
    #pragma omp parallel for collapse(2)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t g = 0; g < groups; g++) {
            const uint16_t* a = o + (r * groups + g) * gd;
            for (int64_t j = 0; j < rank; j++) {
                const uint16_t* b = w + (g * rank + j) * gd;
                float acc = 0.0f;
                for (int64_t c = 0; c < gd; c++)
                    acc += orc_bf16_to_f32(a[c]) * orc_bf16_to_f32(b[c]);
                h[(r * groups + g) * rank + j] = orc_f32_to_bf16(acc);
            }
        }
}

/* bf16 <-> f32 bulk helpers for the Python side */
void orc_f32_to_bf16_n(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_bf16(x[i]);
}
void orc_f32_to_e4m3_n(const float* x, uint8_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_e4m3(x[i]);
}
