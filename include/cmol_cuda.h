/*
 * cmol_cuda.h — additive extensions of the libcmol API for the B200 engine.
 *
 * Nothing here changes cmol.h; every declaration is new.  These are the
 * entry points a token-id workload, a multi-GPU deployment or a benchmark
 * needs and that the text-only reference API (include/cmol.h:219-223 of
 * nvlass/libcmol) cannot express.
 */
#ifndef CMOL_CUDA_H
#define CMOL_CUDA_H

#include "cmol.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device selection ----------------------------------------------------
 * GPUs used by the next cmol_load on any thread.  Sessions are spread over
 * them at acquire time (weights are replicated, no inter-GPU traffic).
 * Default: the environment variable CMOL_CUDA_DEVICES ("0,1,2"), else
 * device 0.  Returns CMOL_ERR_ARGS for an invalid list. */
cmol_err_t cmol_cuda_set_devices(const int *devices, int n);

/* Engine knobs for the next cmol_load (0 keeps the default).
 *   kv_page_tokens : tokens per KV page (default 64: one kv head's K and V of a
 *                    page form one contiguous block, which attention reads
 *                    at full HBM rate; much smaller pages read far slower)
 *   kv_pool_frac   : fraction of free device memory the KV pool may take
 *                    when the full max_sessions * max_ctx does not fit
 *                    (default 0.85)
 *   max_batch      : most sessions in one decode step (default max_sessions)
 *   use_graphs     : 1 = capture the decode step in a CUDA graph (default),
 *                    0 = launch kernels directly (debugging)
 *   kv_dtype       : KV cache format, 0 = f32 (the reference's own,
 *                    src/cmol_internal.h:142-147; default), 1 = f16 (every
 *                    K and V value rounded to the nearest f16 when written:
 *                    half the KV memory and attention traffic; logits stay
 *                    within the engine's 2e-2 / cosine 0.9999 tolerance) */
typedef struct {
    int   kv_page_tokens;
    float kv_pool_frac;
    int   max_batch;
    int   use_graphs;
    int   kv_dtype;
} cmol_cuda_options_t;
void cmol_cuda_set_options(const cmol_cuda_options_t *opt);

/* ---- token-id generation -------------------------------------------------
 * cmol_generate with token ids in place of text: the same prefill, sampling,
 * repeat window, stop rules and callback semantics (src/api.c:437-521 of the
 * reference), minus the tokenizer step.  The callback receives ids. */
typedef int (*cmol_id_cb_t)(int32_t token, int is_eos, void *userdata);

cmol_err_t cmol_generate_ids(cmol_session_t          *s,
                             const int32_t           *prompt,
                             int                      n_prompt,
                             const cmol_gen_params_t *params,
                             cmol_id_cb_t             on_token,
                             void                    *userdata);

/* Many sessions at once from one thread: all items are admitted to the
 * batchers together and the call returns when every item has finished.
 * Generated ids go to out[0..n_out) (at most out_cap); `status` is the
 * per-item cmol_generate_ids result.  Items must use distinct sessions. */
typedef struct {
    cmol_session_t          *session;
    const int32_t           *prompt;
    int                      n_prompt;
    const cmol_gen_params_t *params;
    int32_t                 *out;
    int                      out_cap;
    int                      n_out;      /* set by the call */
    cmol_err_t               status;     /* set by the call */
} cmol_batch_item_t;

cmol_err_t cmol_generate_batch(cmol_batch_item_t *items, int n_items);

/* ---- teacher forcing / introspection -------------------------------------
 * Run one token at the session's next position and copy the logits
 * [vocab] out (the analogue of cmol_model_forward, src/model.h:21-24). */
cmol_err_t cmol_forward_logits(cmol_session_t *s, int32_t token, float *logits_out);

/* Teacher forcing for n sessions in ONE decode step (n columns): session
 * ss[i] runs tokens[i] at its next position and logits_out[i*vocab ..
 * (i+1)*vocab) receives its logits.  The sessions must be distinct and on
 * one GPU (cmol_session_device), n at most that GPU's step width (the
 * model's max_sessions share plus its prefill chunk).  A step of 16 or more
 * columns runs the tensor-core matmuls, so this is how a test checks the
 * wide-batch path logit by logit. */
cmol_err_t cmol_forward_logits_batch(cmol_session_t *const *ss, const int32_t *tokens, int n,
                                     float *logits_out);

int cmol_session_n_tokens(const cmol_session_t *s);
int cmol_session_device(const cmol_session_t *s);

/* Session KV snapshots for multi-turn reuse (call between requests, with no
 * request of the session in flight).
 *   cmol_cuda_session_save: writes the session's context (its token count and
 *     the K and V of every cached position, all layers, in the engine's KV
 *     format) to buf and its size to *size; with buf NULL only the size.
 *     CMOL_ERR_TRUNC when cap is smaller than the size.
 *   cmol_cuda_session_restore: loads a snapshot into a session of a model
 *     with the same layer count, vocabulary, KV format and page size (on any
 *     of its GPUs): the session continues from that context, as if it had
 *     run those tokens.  CMOL_ERR_INVALID for a snapshot of another shape,
 *     CMOL_ERR_CTX_FULL past the model's context, CMOL_ERR_OOM when its GPU
 *     has no free KV pages left.  The weights are not compared: restoring a
 *     snapshot taken with another model of the same shapes gives that
 *     model's context. */
cmol_err_t cmol_cuda_session_save(cmol_session_t *s, void *buf, size_t cap, size_t *size);
cmol_err_t cmol_cuda_session_restore(cmol_session_t *s, const void *buf, size_t size);
int cmol_vocab_size(const cmol_model_t *m);
int cmol_eos_id(const cmol_model_t *m);

/* ---- measurement ---------------------------------------------------------
 * Per-GPU counters since load or the last reset.  decode_ms is device time
 * between CUDA events recorded on the engine stream around every decode
 * step; weight_bytes is the GGUF bytes of all matrices one step streams. */
typedef struct {
    long long decode_steps;
    long long decode_tokens;     /* sampled tokens                        */
    long long prefill_tokens;    /* prompt tokens run through the model   */
    double    decode_ms;
    double    step_ms_last;
    long long weight_bytes;
    long long kv_bytes_read;     /* KV bytes the attention read (sum)     */
    int       kernel_launches_per_step;
    int       graph_steps;       /* steps run through a CUDA graph        */
    long long steps;             /* all steps (prefill, decode and mixed) */
    double    step_ms_total;     /* device time of all steps              */
    unsigned  last_fault_code;   /* device fault word of the last failed
                                    step (0: none since load): 1/2 GEMV
                                    pipeline wait, 3 token id outside the
                                    vocabulary, 4 page outside the pool,
                                    5 sampler found no finite candidate,
                                    6 attention page wait, 7 planted
                                    wait (cmol_cuda_debug_inject 3)     */
    long long h2d_bytes_per_step;   /* host -> device bytes one step copies
                                       (its metadata)                    */
    long long d2h_bytes_per_step;   /* device -> host bytes one step copies
                                       (sampled ids and the fault word)  */
} cmol_cuda_stats_t;

cmol_err_t cmol_cuda_stats(const cmol_model_t *m, int gpu_index, cmol_cuda_stats_t *out);

/* The GEMV launches of one single-session decode step (every weight matrix
 * streamed once) replayed `reps` times alone from a CUDA graph on GPU
 * `gpu_index`; device milliseconds per pass from CUDA events, the GGUF bytes
 * of the matrices and the number of launches per pass.  Must not overlap a
 * generation on that GPU (CMOL_ERR_NO_SESSION if one is running). */
cmol_err_t cmol_cuda_gemv_sweep(cmol_model_t *m, int gpu_index, int reps, double *ms_per_pass,
                                long long *bytes_per_pass, int *launches_per_pass);
void       cmol_cuda_stats_reset(cmol_model_t *m);

/* One kernel class of the widest step run on GPU `gpu_index` since load or
 * the last cmol_cuda_stats_reset (the latest of equal width), replayed alone
 * `reps` times from a CUDA graph; device milliseconds per pass (CUDA events
 * on the engine stream), algorithmic bytes and flops per pass, launches per
 * pass.  Must not overlap a generation on that GPU (CMOL_ERR_NO_SESSION).
 *   CMOL_CUDA_SWEEP_MATMUL    : every weight product of the step at its
 *                               width, no KV written; bytes = GGUF bytes of
 *                               the matrices, flops = 2 * weights * columns;
 *   CMOL_CUDA_SWEEP_ATTENTION : the step's attention over the same sessions
 *                               and positions (reads the KV cache only);
 *                               bytes = K and V bytes at those positions. */
#define CMOL_CUDA_SWEEP_MATMUL 0
#define CMOL_CUDA_SWEEP_ATTENTION 1
cmol_err_t cmol_cuda_kernel_sweep(cmol_model_t *m, int gpu_index, int what, int reps, double *ms_per_pass,
                                  long long *bytes_per_pass, double *flops_per_pass, int *launches_per_pass);

/* Fault-path test hook.  The next decode step on GPU `gpu_index` carries a
 * planted error that the kernels' own bounds checks catch, record in the
 * device fault word and skip (no out-of-range access happens):
 *   kind 1: column 0's token id is vocab + 3 (code 3);
 *   kind 2: a page-table update names a page past the pool (code 4);
 *   kind 3: the step's first kernel waits on a barrier that nothing arrives
 *           on until its bounded wait runs out (a few ms; code 7), as any
 *           device wait does when an arrival is lost.
 * That step fails: the requests in it return CMOL_ERR_INVALID, and
 * cmol_cuda_stats reports the code.  Later steps run normally. */
cmol_err_t cmol_cuda_debug_inject(cmol_model_t *m, int gpu_index, int kind);
int        cmol_cuda_n_gpus(const cmol_model_t *m);

#ifdef __cplusplus
}
#endif
#endif /* CMOL_CUDA_H */
