/*
 * cmol_oracle.h — CPU restatement of the libcmol decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * engine in libcmol_b200/ is compared against; it is never linked into,
 * loaded by, or called from the product.  Only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py may
 * use it.
 *
 * Every function restates the arithmetic of the reference (nvlass/libcmol)
 * in plain C99, citing the reference file:line it follows.  The dot-product
 * kernel can run in two accumulation orders:
 *   lanes == 1  : strictly sequential, as cmol_matmul_scalar (src/quant.c:334-376)
 *   lanes == 16 : sixteen interleaved fused-multiply-add lanes reduced in the
 *                 order of GCC's _mm512_reduce_add_ps, as cmol_matmul_avx512
 *                 (src/quant.c:488-566), the kernel the reference selects on an
 *                 AVX-512 host (src/quant.c:676-705).
 *
 * Q4_0 is NOT implemented by the reference (src/quant.c:298-308 returns 0 for
 * it).  The Q4_0 block decode here follows the GGUF/ggml block format
 * (18 bytes: f16 d, 16 bytes of nibbles; value j = d*((qs[j]&15)-8),
 * value j+16 = d*((qs[j]>>4)-8)) and is pinned against gguf-py 0.19.0's
 * dequantize, not against the reference.
 *
 * Parity pins: tests/test_oracle.py checks this library against the
 * reference's own known-answer vectors (tests/test_quant.c,
 * tests/test_model.c, tests/test_sampler.c of the reference) and against the
 * committed golden fixtures under tests/golden/, which were produced by the
 * reference itself built from its sources (oracle/Makefile, target "ref").
 */
#ifndef CMOL_ORACLE_H
#define CMOL_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF type tags, same numbering as src/cmol_internal.h:27-37. */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q4_0 = 2, ORC_Q5_0 = 6, ORC_Q8_0 = 8,
    ORC_Q4_K = 12, ORC_Q6_K = 14
};

/* Values per block and bytes per block; 0 for an unknown tag. */
int    orc_block_values(int dtype);
size_t orc_block_bytes(int dtype);
size_t orc_row_bytes(int k, int dtype);

float orc_f16_to_f32(uint16_t h);

/* src/quant.c:241-289 (+ Q4_0 from the GGUF format). */
void orc_dequant_row(const void *src, float *dst, int n, int dtype);

/* out[mi*n+ni] = sum_k deq(A[mi,k]) * b[k*n+ni]   (src/quant.c:334-566) */
void orc_matmul(float *out, const void *a, const float *b,
                int m, int k, int n, int dtype, int lanes);

/* src/model.c:90-166 */
void orc_rms_norm(const float *x, const float *w, float *out, int n, float eps);
void orc_softmax(float *x, int n);
void orc_swiglu(const float *gate, const float *up, float *out, int n);
void orc_rope_apply(float *q, float *k, int pos, int n_heads, int n_kv_heads,
                    int head_dim, float freq_base);

/* ---- model ------------------------------------------------------------ */

typedef struct {
    const void *data;   /* packed GGUF bytes, NULL = absent */
    int         dtype;
} orc_tensor_t;

typedef struct {
    int   n_layers, n_heads, n_kv_heads, d_model, d_head, d_ffn, vocab_size;
    float rope_freq_base, rms_norm_eps;
    int   no_rope_layer_interval;
    int   matmul_lanes;              /* 1 or 16, see file header           */
    orc_tensor_t token_embd, output_norm, output;   /* output.data NULL: tied */
    /* per-layer arrays of n_layers entries */
    orc_tensor_t *attn_norm, *attn_q, *attn_k, *attn_v, *attn_output;
    orc_tensor_t *attn_q_norm, *attn_k_norm;        /* entries may be absent  */
    orc_tensor_t *ffn_norm, *ffn_gate, *ffn_up, *ffn_down;
} orc_model_t;

typedef struct orc_session orc_session_t;

orc_session_t *orc_session_new(const orc_model_t *m, int max_ctx);
void           orc_session_free(orc_session_t *s);
void           orc_session_reset(orc_session_t *s);
/* Study switch (not in the reference): store K and V rounded to f16. */
void           orc_set_kv_f16(int on);
int            orc_session_n_tokens(const orc_session_t *s);

/* One token through the whole stack (src/model.c:176-276, src/attn.c:27-146).
 * Returns the logits [vocab_size] inside the session scratch, or NULL. */
float *orc_forward(const orc_model_t *m, orc_session_t *s, int32_t token, int pos);

/* ---- sampler (src/sampler.c) ------------------------------------------ */

typedef struct {
    float        temperature;
    float        top_p;
    int          top_k;
    int          max_new_tokens;
    unsigned int seed;
    float        repeat_penalty;
    int          repeat_last_n;
} orc_params_t;                      /* same layout as cmol_gen_params_t */

void     orc_rng_seed(uint64_t state[4], unsigned int seed);
uint64_t orc_rng_next(uint64_t state[4]);
void     orc_apply_repeat_penalty(float *logits, int vocab_size,
                                  const int32_t *tokens, int n_tokens, float penalty);
int32_t  orc_sample(float *logits, int vocab_size, const orc_params_t *p,
                    uint64_t *rng_state);

/* The id-level generate loop of src/api.c:437-521: clamp the prompt to the
 * free context, prefill, seed the RNG, seed the repeat ring from the prompt
 * tail, then sample / stop / forward.  Writes generated ids to out_ids
 * (at most out_cap) and, when logits_out is not NULL, the logits each
 * sampled token was drawn from (before penalty/temperature, vocab floats per
 * step, at most logits_cap steps).  eos_id < 0 disables the EOS stop.
 * Returns the number of ids written, or a negative code:
 *   -7 context already full, -3 forward failed. */
int orc_generate_ids(const orc_model_t *m, orc_session_t *s,
                     const int32_t *prompt, int n_prompt,
                     const orc_params_t *p, int32_t eos_id,
                     int32_t *out_ids, int out_cap,
                     float *logits_out, int logits_cap);

#ifdef __cplusplus
}
#endif
#endif /* CMOL_ORACLE_H */
