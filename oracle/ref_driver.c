/*
 * ref_driver.c — token-id level driver around the UNMODIFIED reference.
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY.  Compiled together with the
 * reference's own unity source (src/cmol.c of nvlass/libcmol) by
 * oracle/Makefile into oracle/_ref/libcmolref.so.  It calls the reference's
 * exported internals the same way the reference's tests do
 * (tests/test_model_ref.c:165,208): cmol_model_forward, cmol_sample,
 * cmol_apply_repeat_penalty, cmol_rng_seed, cmol_kernels_select,
 * cmol_matmul_scalar, cmol_dequant_row.  Nothing in the product links it.
 */
#include "cmol_internal.h"
#include "model.h"
#include "quant.h"
#include "sampler.h"

#include <string.h>

const char *ref_kernel_name(void) { return cmol_kernels_select().name; }

void ref_dequant_row(const void *src, float *dst, int n, int dtype) {
    cmol_dequant_row(src, dst, n, (cmol_dtype_t)dtype);
}

/* which: 0 = scalar kernel, 1 = the kernel cmol_kernels_select() picks */
void ref_matmul(float *out, const void *a, const float *b,
                int m, int k, int n, int dtype, int which) {
    if (which) cmol_kernels_select().matmul(out, a, b, m, k, n, (cmol_dtype_t)dtype);
    else       cmol_matmul_scalar(out, a, b, m, k, n, (cmol_dtype_t)dtype);
}

void ref_rms_norm(const float *x, const float *w, float *out, int n, float eps) {
    cmol_rms_norm(x, w, out, n, eps);
}
void ref_rope_apply(float *q, float *k, int pos, int nh, int nkv, int hd, float base) {
    cmol_rope_apply(q, k, pos, nh, nkv, hd, base);
}
void ref_swiglu(const float *g, const float *u, float *o, int n) { cmol_swiglu(g, u, o, n); }
void ref_softmax(float *x, int n) { cmol_softmax(x, n); }

void     ref_rng_seed(uint64_t st[4], unsigned int seed) { cmol_rng_seed(st, seed); }
uint64_t ref_rng_next(uint64_t st[4]) { return cmol_rng_next(st); }
void     ref_repeat_penalty(float *l, int V, const int32_t *t, int n, float p) {
    cmol_apply_repeat_penalty(l, V, t, n, p);
}
int32_t  ref_sample(float *logits, int V, const cmol_gen_params_t *p, uint64_t *rng) {
    return cmol_sample(logits, V, p, rng);
}

int  ref_vocab_size(cmol_model_t *m) { return m->hparams.vocab_size; }
int  ref_eos_id(cmol_model_t *m) { return m->tokenizer.eos_id; }
int  ref_n_tokens(cmol_session_t *s) { return s->kvcache.n_tokens; }
int  ref_max_tokens(cmol_session_t *s) { return s->kvcache.max_tokens; }
void ref_set_n_tokens(cmol_session_t *s, int n) { s->kvcache.n_tokens = n; }

/* Teacher-forcing step: one token at `pos`; copies the logits out. */
int ref_forward(cmol_model_t *m, cmol_session_t *s, int32_t tok, int pos, float *logits_out) {
    float *l = cmol_model_forward(m, s, tok, pos);
    if (!l) return -3;
    if (pos + 1 > s->kvcache.n_tokens) s->kvcache.n_tokens = pos + 1;
    if (logits_out) memcpy(logits_out, l, (size_t)m->hparams.vocab_size * sizeof(float));
    return 0;
}

/* The generate loop of src/api.c:437-521 with token ids in place of text
 * (the tokenizer step of api.c:430-435 is skipped).  Semantics as
 * orc_generate_ids in cmol_oracle.h. */
int ref_generate_ids(cmol_session_t *s, const int32_t *prompt, int n_prompt,
                     const cmol_gen_params_t *p, int32_t eos_id,
                     int32_t *out_ids, int out_cap, float *logits_out, int logits_cap) {
    cmol_model_t *m = s->model;
    int V = m->hparams.vocab_size;
    if (s->kvcache.n_tokens >= s->kvcache.max_tokens) return CMOL_ERR_CTX_FULL;
    if (n_prompt <= 0) return 0;
    int avail = s->kvcache.max_tokens - s->kvcache.n_tokens;
    if (n_prompt > avail) n_prompt = avail;

    float *logits = NULL;
    int pos = s->kvcache.n_tokens;
    for (int i = 0; i < n_prompt; i++) logits = cmol_model_forward(m, s, prompt[i], pos++);
    s->kvcache.n_tokens = pos;
    if (!logits) return CMOL_ERR_INVALID;

    int max_new = p->max_new_tokens;
    if (max_new < 0) max_new = s->kvcache.max_tokens;
    uint64_t rng[4];
    cmol_rng_seed(rng, p->seed);

    int32_t ring[CMOL_REPEAT_BUF];
    int last_n = p->repeat_last_n;
    if (last_n <= 0 || last_n > CMOL_REPEAT_BUF) last_n = CMOL_REPEAT_BUF;
    int seed_n = n_prompt < last_n ? n_prompt : last_n;
    for (int i = 0; i < seed_n; i++) ring[i] = prompt[n_prompt - seed_n + i];
    int head = seed_n % CMOL_REPEAT_BUF, fill = seed_n;

    int n_out = 0, n_gen = 0, step = 0;
    for (;;) {
        if (logits_out && step < logits_cap)
            memcpy(logits_out + (size_t)step * V, logits, (size_t)V * sizeof(float));
        step++;
        if (p->repeat_penalty > 1.0f && fill > 0)
            cmol_apply_repeat_penalty(logits, V, ring, fill, p->repeat_penalty);
        int32_t next = cmol_sample(logits, V, p, rng);
        int is_eos = eos_id >= 0 && next == eos_id;
        if (n_out < out_cap) out_ids[n_out] = next;
        n_out++;
        if (is_eos) break;
        ring[head] = next;
        head = (head + 1) % CMOL_REPEAT_BUF;
        if (fill < CMOL_REPEAT_BUF) fill++;
        n_gen++;
        if (max_new > 0 && n_gen >= max_new) break;
        if (pos >= s->kvcache.max_tokens) break;
        logits = cmol_model_forward(m, s, next, pos++);
        s->kvcache.n_tokens = pos;
        if (!logits) return CMOL_ERR_INVALID;
    }
    return n_out < out_cap ? n_out : out_cap;
}
