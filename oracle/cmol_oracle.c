/*
 * cmol_oracle.c — CPU restatement of the libcmol decode path.
 * TEST INFRASTRUCTURE ONLY (see cmol_oracle.h); never part of the product.
 *
 * Build with -std=c99 -ffp-contract=off so that every multiply and add is
 * rounded separately, exactly as the reference's scalar code is compiled
 * (ISO C mode disables contraction in GCC); the only fused operations are
 * the explicit fmaf() calls that restate _mm512_fmadd_ps.
 */
#include "cmol_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

/* ------------------------------------------------------------------------
 * f16 -> f32.  Exact for every half value (normal, subnormal, inf, nan),
 * which is all src/quant.c:38-63 computes.  Written as a scaled integer
 * here rather than by re-assembling exponent bits.
 * --------------------------------------------------------------------- */
float orc_f16_to_f32(uint16_t h) {
    int   sign = (h >> 15) & 1;
    int   e    = (h >> 10) & 0x1F;
    int   mant = h & 0x3FF;
    float v;
    if (e == 0x1F) {
        v = mant ? NAN : INFINITY;
    } else if (e == 0) {
        v = ldexpf((float)mant, -24);                 /* subnormal / zero */
    } else {
        v = ldexpf((float)(mant | 0x400), e - 25);    /* 1.m * 2^(e-15)   */
    }
    return sign ? -v : v;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

int orc_block_values(int dtype) {
    switch (dtype) {
    case ORC_F32: case ORC_F16: return 1;
    case ORC_Q4_0: case ORC_Q5_0: case ORC_Q8_0: return 32;
    case ORC_Q4_K: case ORC_Q6_K: return 256;
    default: return 0;
    }
}

size_t orc_block_bytes(int dtype) {
    switch (dtype) {
    case ORC_F32:  return 4;
    case ORC_F16:  return 2;
    case ORC_Q4_0: return 18;
    case ORC_Q5_0: return 22;
    case ORC_Q8_0: return 34;
    case ORC_Q4_K: return 144;
    case ORC_Q6_K: return 210;
    default: return 0;
    }
}

size_t orc_row_bytes(int k, int dtype) {
    int bv = orc_block_values(dtype);
    if (!bv) return 0;
    return (size_t)(k / bv) * orc_block_bytes(dtype);
}

/* ------------------------------------------------------------------------
 * Block decoders.  Byte offsets follow the packed structs of
 * src/quant.c:78-105; formulas follow src/quant.c:152-232.
 * --------------------------------------------------------------------- */

/* Q8_0: f16 d, int8 qs[32]   (src/quant.c:85-89, 166-170) */
static void blk_q8_0(const uint8_t *b, float *dst) {
    float d = orc_f16_to_f32(rd16(b));
    const int8_t *qs = (const int8_t *)(b + 2);
    for (int i = 0; i < 32; i++) dst[i] = d * (float)qs[i];
}

/* Q5_0: f16 d, u8 qh[4], u8 qs[16]   (src/quant.c:78-83, 152-164) */
static void blk_q5_0(const uint8_t *b, float *dst) {
    float    d  = orc_f16_to_f32(rd16(b));
    uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) |
                  ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    const uint8_t *qs = b + 6;
    for (int j = 0; j < 16; j++) {
        int lo = (qs[j] & 0x0F) | (int)(((qh >> j) & 1u) << 4);
        int hi = (qs[j] >> 4)   | (int)(((qh >> (j + 16)) & 1u) << 4);
        dst[j]      = d * (float)(lo - 16);
        dst[j + 16] = d * (float)(hi - 16);
    }
}

/* Q4_0 (GGUF format; not implemented by the reference): f16 d, u8 qs[16] */
static void blk_q4_0(const uint8_t *b, float *dst) {
    float d = orc_f16_to_f32(rd16(b));
    const uint8_t *qs = b + 2;
    for (int j = 0; j < 16; j++) {
        dst[j]      = d * (float)((qs[j] & 0x0F) - 8);
        dst[j + 16] = d * (float)((qs[j] >> 4) - 8);
    }
}

/* Q4_K 6-bit scale/min unpack   (src/quant.c:125-134) */
static void q4k_scale_min(int j, const uint8_t *s, int *sc, int *mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4)   | ((s[j]     >> 6) << 4);
    }
}

/* Q4_K: f16 d, f16 dmin, u8 scales[12], u8 qs[128]  (src/quant.c:91-97, 172-194) */
static void blk_q4_k(const uint8_t *b, float *dst) {
    float d    = orc_f16_to_f32(rd16(b));
    float dmin = orc_f16_to_f32(rd16(b + 2));
    const uint8_t *sc12 = b + 4;
    const uint8_t *qs   = b + 16;
    for (int sub = 0; sub < 8; sub++) {
        int sc, mn;
        q4k_scale_min(sub, sc12, &sc, &mn);
        float db = d * (float)sc;
        float mb = dmin * (float)mn;
        const uint8_t *q = qs + (sub / 2) * 32;
        int shift = (sub & 1) ? 4 : 0;
        for (int l = 0; l < 32; l++)
            dst[sub * 32 + l] = db * (float)((q[l] >> shift) & 0xF) - mb;
    }
}

/* Q6_K: u8 ql[128], u8 qh[64], i8 scales[16], f16 d  (src/quant.c:99-105, 196-232) */
static void blk_q6_k(const uint8_t *b, float *dst) {
    const uint8_t *ql = b;
    const uint8_t *qh = b + 128;
    const int8_t  *sc = (const int8_t *)(b + 192);
    float d = orc_f16_to_f32(rd16(b + 208));
    for (int i = 0; i < 256; i++) {
        int g  = i >> 5, j = i & 31;
        int lo = (ql[(g < 4 ? 0 : 64) + (g & 1) * 32 + j] >> ((g & 2) ? 4 : 0)) & 0xF;
        int hi = (qh[(g < 4 ? 0 : 32) + j] >> ((g & 3) * 2)) & 0x3;
        int q  = (lo | (hi << 4)) - 32;
        dst[i] = d * (float)sc[i >> 4] * (float)q;
    }
}

static void dequant_block(const uint8_t *blk, float *tmp, int dtype) {
    switch (dtype) {
    case ORC_Q4_0: blk_q4_0(blk, tmp); break;
    case ORC_Q5_0: blk_q5_0(blk, tmp); break;
    case ORC_Q8_0: blk_q8_0(blk, tmp); break;
    case ORC_Q4_K: blk_q4_k(blk, tmp); break;
    case ORC_Q6_K: blk_q6_k(blk, tmp); break;
    default: break;
    }
}

/* src/quant.c:241-289: NULL / n<=0 / unknown tag leave dst untouched. */
void orc_dequant_row(const void *src, float *dst, int n, int dtype) {
    if (!src || !dst || n <= 0) return;
    const uint8_t *s = (const uint8_t *)src;
    if (dtype == ORC_F32) { memcpy(dst, src, (size_t)n * 4); return; }
    if (dtype == ORC_F16) {
        for (int i = 0; i < n; i++) dst[i] = orc_f16_to_f32(rd16(s + 2 * i));
        return;
    }
    int bv = orc_block_values(dtype);
    if (bv <= 1) return;
    size_t bb = orc_block_bytes(dtype);
    for (int bi = 0; bi < n / bv; bi++) dequant_block(s + bi * bb, dst + bi * bv, dtype);
}

/* ------------------------------------------------------------------------
 * Dot-product kernel.
 * --------------------------------------------------------------------- */

/* Reduction order of GCC's _mm512_reduce_add_ps: halves of 8, then 4, then
 * the pairs {0,2},{1,3}, then the final pair. */
static float reduce16(const float a[16]) {
    float t[8], u[4];
    for (int i = 0; i < 8; i++) t[i] = a[8 + i] + a[i];
    for (int i = 0; i < 4; i++) u[i] = t[4 + i] + t[i];
    float v0 = u[0] + u[2];
    float v1 = u[1] + u[3];
    return v0 + v1;
}

void orc_matmul(float *out, const void *a, const float *b,
                int m, int k, int n, int dtype, int lanes) {
    int bv = orc_block_values(dtype);
    if (!bv || !out || !a || !b) return;
    const uint8_t *ab  = (const uint8_t *)a;
    size_t         rb  = orc_row_bytes(k, dtype);
    float          tmp[256];

    for (int mi = 0; mi < m; mi++) {
        const uint8_t *row = ab + (size_t)mi * rb;
        for (int ni = 0; ni < n; ni++) {
            if (dtype == ORC_F16 || lanes != 16) {
                /* sequential: src/quant.c:345-374 (and the F16 branch of
                 * every SIMD kernel, src/quant.c:527-534) */
                float acc = 0.0f;
                if (dtype == ORC_F32) {
                    const float *af = (const float *)row;
                    for (int ki = 0; ki < k; ki++) acc += af[ki] * b[ki * n + ni];
                } else if (dtype == ORC_F16) {
                    for (int ki = 0; ki < k; ki++)
                        acc += orc_f16_to_f32(rd16(row + 2 * ki)) * b[ki * n + ni];
                } else {
                    for (int bi = 0; bi < k / bv; bi++) {
                        dequant_block(row + bi * orc_block_bytes(dtype), tmp, dtype);
                        for (int j = 0; j < bv; j++)
                            acc += tmp[j] * b[(bi * bv + j) * n + ni];
                    }
                }
                out[mi * n + ni] = acc;
                continue;
            }
            /* sixteen FMA lanes: src/quant.c:503-564 */
            float acc[16] = {0};
            if (dtype == ORC_F32) {
                const float *af = (const float *)row;
                int ki;
                for (ki = 0; ki + 15 < k; ki += 16)
                    for (int l = 0; l < 16; l++)
                        acc[l] = fmaf(af[ki + l], b[(ki + l) * n + ni], acc[l]);
                float tail = reduce16(acc);
                for (; ki < k; ki++) tail += af[ki] * b[ki * n + ni];
                out[mi * n + ni] = tail;
                continue;
            }
            for (int bi = 0; bi < k / bv; bi++) {
                int base = bi * bv;
                dequant_block(row + bi * orc_block_bytes(dtype), tmp, dtype);
                for (int j = 0; j + 15 < bv; j += 16)
                    for (int l = 0; l < 16; l++)
                        acc[l] = fmaf(tmp[j + l], b[(base + j + l) * n + ni], acc[l]);
            }
            out[mi * n + ni] = reduce16(acc);
        }
    }
}

/* ------------------------------------------------------------------------
 * Primitive ops (src/model.c:90-166)
 * --------------------------------------------------------------------- */

void orc_rms_norm(const float *x, const float *w, float *out, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = w[i] * (x[i] * ss);
}

void orc_softmax(float *x, int n) {
    float mx = x[0], sm = 0.0f;
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sm += x[i]; }
    sm = 1.0f / sm;
    for (int i = 0; i < n; i++) x[i] *= sm;
}

void orc_swiglu(const float *gate, const float *up, float *out, int n) {
    for (int i = 0; i < n; i++) {
        float g = gate[i];
        out[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

static void rope_heads(float *v, int pos, int heads, int hd, float base) {
    int half = hd / 2;
    for (int h = 0; h < heads; h++) {
        float *p = v + h * hd;
        for (int i = 0; i < half; i++) {
            float theta = (float)pos / powf(base, (float)(2 * i) / (float)hd);
            float c = cosf(theta), s = sinf(theta);
            float a0 = p[2 * i], a1 = p[2 * i + 1];
            p[2 * i]     = a0 * c - a1 * s;
            p[2 * i + 1] = a0 * s + a1 * c;
        }
    }
}

void orc_rope_apply(float *q, float *k, int pos, int n_heads, int n_kv_heads,
                    int head_dim, float freq_base) {
    rope_heads(q, pos, n_heads, head_dim, freq_base);
    rope_heads(k, pos, n_kv_heads, head_dim, freq_base);
}

/* ------------------------------------------------------------------------
 * Session + forward
 * --------------------------------------------------------------------- */

struct orc_session {
    float *k, *v;          /* [layer][max_tokens][kv_dim], src/cmol_internal.h:137-147 */
    int    max_tokens;
    int    n_tokens;
    float *scratch;
};

orc_session_t *orc_session_new(const orc_model_t *m, int max_ctx) {
    orc_session_t *s = (orc_session_t *)calloc(1, sizeof *s);
    if (!s) return NULL;
    size_t kvd = (size_t)m->n_kv_heads * m->d_head;
    size_t kv  = (size_t)m->n_layers * max_ctx * kvd;
    size_t scr = 5u * m->d_model + 2u * kvd + (size_t)max_ctx + 2u * m->d_ffn + m->vocab_size;
    s->k = (float *)calloc(kv, 4);
    s->v = (float *)calloc(kv, 4);
    s->scratch = (float *)calloc(scr, 4);
    s->max_tokens = max_ctx;
    if (!s->k || !s->v || !s->scratch) { orc_session_free(s); return NULL; }
    return s;
}

/* Not part of the reference: an f16 KV format (the engine stores f32, as
 * the reference does).  With orc_set_kv_f16(1) every K and V value is
 * rounded to the nearest f16 (ties to even, the compiler's _Float16
 * conversion) when written, so the effect of such a format on the logits
 * can be measured against the f32 cache. */
static int g_kv_f16 = 0;
void orc_set_kv_f16(int on) { g_kv_f16 = on != 0; }
static float kv_round_f16(float x) { return (float)(_Float16)x; }

void orc_session_free(orc_session_t *s) {
    if (!s) return;
    free(s->k); free(s->v); free(s->scratch); free(s);
}

void orc_session_reset(orc_session_t *s) { if (s) s->n_tokens = 0; }
int  orc_session_n_tokens(const orc_session_t *s) { return s ? s->n_tokens : 0; }

static void mm(const orc_model_t *m, float *out, const orc_tensor_t *t,
               const float *x, int rows, int k) {
    orc_matmul(out, t->data, x, rows, k, 1, t->dtype, m->matmul_lanes);
}

/* src/attn.c:27-146 */
static void attn_forward(const orc_model_t *m, orc_session_t *s, int L, int pos,
                         const float *xnorm, float *q, float *kb, float *vb,
                         float *scores, float *out) {
    int nh = m->n_heads, nkv = m->n_kv_heads, hd = m->d_head, d = m->d_model;
    int kvd = nkv * hd;

    mm(m, q,  &m->attn_q[L], xnorm, d,   d);
    mm(m, kb, &m->attn_k[L], xnorm, kvd, d);
    mm(m, vb, &m->attn_v[L], xnorm, kvd, d);

    if (m->attn_q_norm && m->attn_q_norm[L].data)
        for (int h = 0; h < nh; h++)
            orc_rms_norm(q + h * hd, (const float *)m->attn_q_norm[L].data,
                         q + h * hd, hd, m->rms_norm_eps);
    if (m->attn_k_norm && m->attn_k_norm[L].data)
        for (int h = 0; h < nkv; h++)
            orc_rms_norm(kb + h * hd, (const float *)m->attn_k_norm[L].data,
                         kb + h * hd, hd, m->rms_norm_eps);

    int nope = m->no_rope_layer_interval > 0 && (L + 1) % m->no_rope_layer_interval == 0;
    if (!nope) orc_rope_apply(q, kb, pos, nh, nkv, hd, m->rope_freq_base);

    float *kl = s->k + (size_t)L * s->max_tokens * kvd;
    float *vl = s->v + (size_t)L * s->max_tokens * kvd;
    memcpy(kl + (size_t)pos * kvd, kb, (size_t)kvd * 4);
    memcpy(vl + (size_t)pos * kvd, vb, (size_t)kvd * 4);
    if (g_kv_f16)                     /* study of an f16 KV format: store rounded */
        for (int i = 0; i < kvd; i++) {
            kl[(size_t)pos * kvd + i] = kv_round_f16(kb[i]);
            vl[(size_t)pos * kvd + i] = kv_round_f16(vb[i]);
        }

    float scale = 1.0f / sqrtf((float)hd);
    int   n     = pos + 1;
    memset(out, 0, (size_t)d * 4);
    for (int h = 0; h < nh; h++) {
        int    hk = h * nkv / nh;
        float *qh = q + h * hd, *oh = out + h * hd;
        for (int t = 0; t < n; t++) {
            const float *kt = kl + (size_t)t * kvd + hk * hd;
            float dot = 0.0f;
            for (int i = 0; i < hd; i++) dot += qh[i] * kt[i];
            scores[t] = dot * scale;
        }
        orc_softmax(scores, n);
        for (int t = 0; t < n; t++) {
            const float *vt = vl + (size_t)t * kvd + hk * hd;
            float p = scores[t];
            for (int i = 0; i < hd; i++) oh[i] += p * vt[i];
        }
    }
    memcpy(q, out, (size_t)d * 4);
    mm(m, out, &m->attn_output[L], q, d, d);
}

/* src/model.c:176-276 */
float *orc_forward(const orc_model_t *m, orc_session_t *s, int32_t token, int pos) {
    if (!m || !s || !m->token_embd.data) return NULL;
    int d = m->d_model, kvd = m->n_kv_heads * m->d_head, F = m->d_ffn;
    float *x      = s->scratch;
    float *xn     = x + d;
    float *q      = xn + d;
    float *kb     = q + d;
    float *vb     = kb + kvd;
    float *scores = vb + kvd;
    float *ao     = scores + s->max_tokens;
    float *g      = ao + d;
    float *u      = g + F;
    float *logits = u + F;

    orc_dequant_row((const uint8_t *)m->token_embd.data +
                        (size_t)token * orc_row_bytes(d, m->token_embd.dtype),
                    x, d, m->token_embd.dtype);

    for (int L = 0; L < m->n_layers; L++) {
        orc_rms_norm(x, (const float *)m->attn_norm[L].data, xn, d, m->rms_norm_eps);
        attn_forward(m, s, L, pos, xn, q, kb, vb, scores, ao);
        for (int i = 0; i < d; i++) x[i] += ao[i];

        orc_rms_norm(x, (const float *)m->ffn_norm[L].data, xn, d, m->rms_norm_eps);
        mm(m, g, &m->ffn_gate[L], xn, F, d);
        mm(m, u, &m->ffn_up[L],   xn, F, d);
        orc_swiglu(g, u, g, F);
        mm(m, ao, &m->ffn_down[L], g, d, F);
        for (int i = 0; i < d; i++) x[i] += ao[i];
    }
    orc_rms_norm(x, (const float *)m->output_norm.data, xn, d, m->rms_norm_eps);
    const orc_tensor_t *head = m->output.data ? &m->output : &m->token_embd;
    mm(m, logits, head, xn, m->vocab_size, d);
    return logits;
}

/* ------------------------------------------------------------------------
 * Sampler (src/sampler.c)
 * --------------------------------------------------------------------- */

static uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

/* xoshiro256** step, src/sampler.c:37-49 */
uint64_t orc_rng_next(uint64_t s[4]) {
    uint64_t out = rotl(s[1] * 5u, 7) * 9u;
    uint64_t t   = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3]  = rotl(s[3], 45);
    return out;
}

/* splitmix64 expansion, src/sampler.c:52-75 (seed 0 = time-based, as there) */
static uint64_t splitmix(uint64_t *x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void orc_rng_seed(uint64_t st[4], unsigned int seed) {
    uint64_t x;
    if (seed == 0) {
        static uint64_t ctr = 0;
        x  = (uint64_t)time(NULL);
        x ^= ++ctr * 6364136223846793005ULL;
        x ^= (uint64_t)(uintptr_t)st;
        if (!x) x = 0xDEADBEEFCAFEBABEULL;
    } else {
        x = (uint64_t)seed;
    }
    for (int i = 0; i < 4; i++) st[i] = splitmix(&x);
}

/* uniform [0,1) from the top 23 bits, src/sampler.c:78-84 */
static float rng_unit(uint64_t st[4]) {
    uint32_t bits = 0x3F800000u | (uint32_t)(orc_rng_next(st) >> 41);
    float f;
    memcpy(&f, &bits, 4);
    return f - 1.0f;
}

/* src/sampler.c:171-184 */
void orc_apply_repeat_penalty(float *logits, int V, const int32_t *tok, int n,
                              float penalty) {
    if (penalty <= 1.0f || !logits || !tok || n <= 0) return;
    for (int i = 0; i < n; i++) {
        int32_t id = tok[i];
        if (id < 0 || id >= V) continue;
        if (logits[id] > 0.0f) logits[id] /= penalty;
        else                   logits[id] *= penalty;
    }
}

typedef struct { float val; int32_t idx; } tp_t;

/* min-heap of size <= k, src/sampler.c:107-165 */
static void sift_down(tp_t *h, int i, int n) {
    for (;;) {
        int s = i, l = 2 * i + 1, r = l + 1;
        if (l < n && h[l].val < h[s].val) s = l;
        if (r < n && h[r].val < h[s].val) s = r;
        if (s == i) return;
        tp_t t = h[i]; h[i] = h[s]; h[s] = t;
        i = s;
    }
}

static void sift_up(tp_t *h, int i) {
    while (i > 0) {
        int p = (i - 1) / 2;
        if (h[p].val <= h[i].val) return;
        tp_t t = h[i]; h[i] = h[p]; h[p] = t;
        i = p;
    }
}

static int cmp_desc(const void *a, const void *b) {
    float x = ((const tp_t *)a)->val, y = ((const tp_t *)b)->val;
    return (x < y) ? 1 : (x > y) ? -1 : 0;
}

#define ORC_TOPK_MAX 512   /* src/sampler.c:150 */

int32_t orc_sample(float *logits, int V, const orc_params_t *p, uint64_t *rng) {
    if (!logits || V <= 0) return 0;
    if (!p || p->temperature == 0.0f) {                     /* src/sampler.c:199-204 */
        int32_t best = 0;
        for (int i = 1; i < V; i++) if (logits[i] > logits[best]) best = i;
        return best;
    }
    float inv_t = 1.0f / p->temperature;                    /* 207-210 */
    for (int i = 0; i < V; i++) logits[i] *= inv_t;
    orc_softmax(logits, V);                                 /* 213 */

    int use_k = p->top_k > 0 && p->top_k < V;
    int use_p = p->top_p > 0.0f && p->top_p < 1.0f;
    if (!use_k && !use_p) {                                 /* 219-234 */
        if (!rng) {
            int32_t best = 0;
            for (int i = 1; i < V; i++) if (logits[i] > logits[best]) best = i;
            return best;
        }
        float r = rng_unit(rng), acc = 0.0f;
        for (int i = 0; i < V - 1; i++) {
            acc += logits[i];
            if (r < acc) return i;
        }
        return V - 1;
    }

    tp_t buf[ORC_TOPK_MAX];                                 /* 236-242 */
    int  k = use_k ? p->top_k : V;
    if (k > ORC_TOPK_MAX) k = ORC_TOPK_MAX;
    int  n = 0;
    for (int i = 0; i < V; i++) {
        if (n < k) {
            buf[n].val = logits[i]; buf[n].idx = i;
            sift_up(buf, n);
            n++;
        } else if (logits[i] > buf[0].val) {
            buf[0].val = logits[i]; buf[0].idx = i;
            sift_down(buf, 0, k);
        }
    }
    qsort(buf, (size_t)n, sizeof(tp_t), cmp_desc);

    int nucleus = n;                                        /* 245-253 */
    if (use_p) {
        float cum = 0.0f;
        for (int i = 0; i < n; i++) {
            cum += buf[i].val;
            if (cum >= p->top_p) { nucleus = i + 1; break; }
        }
    }
    float sum = 0.0f;                                       /* 256-267 */
    for (int i = 0; i < nucleus; i++) sum += buf[i].val;
    if (!rng || sum <= 0.0f) return buf[0].idx;
    float r = rng_unit(rng) * sum, acc = 0.0f;
    for (int i = 0; i < nucleus; i++) {
        acc += buf[i].val;
        if (r < acc) return buf[i].idx;
    }
    return buf[nucleus - 1].idx;
}

/* ------------------------------------------------------------------------
 * Generate loop (src/api.c:437-521), token-id level
 * --------------------------------------------------------------------- */

#define ORC_REPEAT_BUF 128   /* src/sampler.h:49 */

int orc_generate_ids(const orc_model_t *m, orc_session_t *s,
                     const int32_t *prompt, int n_prompt,
                     const orc_params_t *p, int32_t eos_id,
                     int32_t *out_ids, int out_cap,
                     float *logits_out, int logits_cap) {
    if (!m || !s || !p || (!prompt && n_prompt > 0)) return -6;
    if (s->n_tokens >= s->max_tokens) return -7;            /* api.c:426 */
    if (n_prompt <= 0) return 0;                            /* api.c:435 */
    int avail = s->max_tokens - s->n_tokens;                /* api.c:438-441 */
    if (n_prompt > avail) n_prompt = avail;

    float *logits = NULL;
    int pos = s->n_tokens;
    for (int i = 0; i < n_prompt; i++) logits = orc_forward(m, s, prompt[i], pos++);
    s->n_tokens = pos;
    if (!logits) return -3;

    int max_new = p->max_new_tokens;
    if (max_new < 0) max_new = s->max_tokens;

    uint64_t rng[4];
    orc_rng_seed(rng, p->seed);

    int32_t ring[ORC_REPEAT_BUF];                           /* api.c:465-476 */
    int last_n = p->repeat_last_n;
    if (last_n <= 0 || last_n > ORC_REPEAT_BUF) last_n = ORC_REPEAT_BUF;
    int seed_n = n_prompt < last_n ? n_prompt : last_n;
    for (int i = 0; i < seed_n; i++) ring[i] = prompt[n_prompt - seed_n + i];
    int head = seed_n % ORC_REPEAT_BUF, fill = seed_n;

    int n_out = 0, n_gen = 0, step = 0;
    for (;;) {
        if (logits_out && step < logits_cap)
            memcpy(logits_out + (size_t)step * m->vocab_size, logits,
                   (size_t)m->vocab_size * 4);
        step++;
        if (p->repeat_penalty > 1.0f && fill > 0)
            orc_apply_repeat_penalty(logits, m->vocab_size, ring, fill, p->repeat_penalty);
        int32_t next = orc_sample(logits, m->vocab_size, p, rng);
        int is_eos = eos_id >= 0 && next == eos_id;
        if (n_out < out_cap) out_ids[n_out] = next;
        n_out++;
        if (is_eos) break;
        ring[head] = next;
        head = (head + 1) % ORC_REPEAT_BUF;
        if (fill < ORC_REPEAT_BUF) fill++;
        n_gen++;
        if (max_new > 0 && n_gen >= max_new) break;
        if (pos >= s->max_tokens) break;
        logits = orc_forward(m, s, next, pos++);
        s->n_tokens = pos;
        if (!logits) return -3;
    }
    return n_out < out_cap ? n_out : out_cap;
}
