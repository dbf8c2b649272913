/*
 * cmol.h — public C API of libcmol, served by the B200 engine.
 *
 * Drop-in contract: every type, enum value, default, struct layout and
 * function signature below is the one of nvlass/libcmol's include/cmol.h
 * (lines 40-316), so code written against that header compiles and links
 * against libcmol.so from this repository unchanged.  The implementation
 * differs: weights live in GPU memory, sessions share a continuous batcher
 * per GPU, and the per-token forward pass runs as CUDA kernels.  Additive,
 * non-breaking extensions (token-id generation, device selection, batch
 * runs) are declared in cmol_cuda.h, not here.
 *
 * Behavioural differences that a caller can observe:
 *   - cmol_load allocates device memory besides the host arena, and fails
 *     with CMOL_ERR_OOM / CMOL_ERR_UNSUPPORTED when no usable GPU exists;
 *   - max_sessions is not capped at 32;
 *   - cmol_arena_estimate returns the host bytes plus the device bytes.
 */

#ifndef CMOL_H
#define CMOL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CMOL_VERSION_MAJOR  0
#define CMOL_VERSION_MINOR  1
#define CMOL_VERSION_PATCH  0
#define CMOL_VERSION_STRING "0.1.0"

/* Negative values are errors; counts are returned as non-negative ints. */
typedef enum {
    CMOL_OK              =  0,
    CMOL_ERR_OOM         = -1, /* host or device memory exhausted          */
    CMOL_ERR_IO          = -2, /* file open / mmap failed                  */
    CMOL_ERR_INVALID     = -3, /* malformed GGUF or missing tensor          */
    CMOL_ERR_UNSUPPORTED = -4, /* unsupported quant type / arch / no GPU    */
    CMOL_ERR_NO_SESSION  = -5, /* session pool exhausted                    */
    CMOL_ERR_ARGS        = -6, /* NULL or out-of-range argument             */
    CMOL_ERR_CTX_FULL    = -7, /* session context full: reset it            */
    CMOL_ERR_TRUNC       = -8, /* output buffer too small                   */
} cmol_err_t;

#define CMOL_LOG_ERROR  0
#define CMOL_LOG_WARN   1
#define CMOL_LOG_INFO   2
#define CMOL_LOG_DEBUG  3

typedef void (*cmol_log_fn_t)(int level, const char *msg, void *userdata);

typedef struct {
    int           max_ctx;       /* context window per session (tokens)   */
    int           max_sessions;  /* session slots                          */
    int           prefill_chunk; /* accepted for compatibility             */
    cmol_log_fn_t log_fn;        /* optional log callback                  */
    void         *log_ud;
} cmol_config_t;

#define CMOL_DEFAULT_CONFIG \
    { .max_ctx = 2048, .max_sessions = 4, .prefill_chunk = 512, \
      .log_fn = NULL, .log_ud = NULL }

typedef struct {
    float        temperature;    /* 0 = greedy                             */
    float        top_p;          /* 1 = off                                */
    int          top_k;          /* 0 = off                                */
    int          max_new_tokens; /* -1 = until EOS or full context         */
    unsigned int seed;           /* 0 = time-based                         */
    float        repeat_penalty; /* 1 = off                                */
    int          repeat_last_n;  /* prompt tail that seeds the window      */
} cmol_gen_params_t;

#define CMOL_DEFAULT_PARAMS \
    { .temperature = 0.8f, .top_p = 0.95f, .top_k = 40, \
      .max_new_tokens = 256, .seed = 0, \
      .repeat_penalty = 1.1f, .repeat_last_n = 64 }

typedef struct cmol_model   cmol_model_t;
typedef struct cmol_session cmol_session_t;

/* Called on the thread that called cmol_generate, once per sampled token.
 * `piece` is not NUL-terminated and is valid only during the call.
 * Return non-zero to stop (cmol_generate still returns CMOL_OK). */
typedef int (*cmol_token_cb_t)(const char *piece, size_t len,
                                int is_eos, void *userdata);

cmol_model_t *cmol_load(const char          *gguf_path,
                         const cmol_config_t *cfg,
                         cmol_err_t          *err);
void cmol_free(cmol_model_t *m);

cmol_session_t *cmol_session_acquire(cmol_model_t *m);
void cmol_session_release(cmol_session_t *s);
void cmol_session_reset(cmol_session_t *s);

cmol_err_t cmol_generate(cmol_session_t          *s,
                          const char              *prompt,
                          const cmol_gen_params_t *params,
                          cmol_token_cb_t          on_token,
                          void                    *userdata);

int cmol_encode(cmol_model_t *m,
                const char   *text,
                int32_t      *out,
                int           out_cap);
const char *cmol_decode_token(cmol_model_t *m, int32_t token_id);

const char *cmol_strerror(cmol_err_t err);
const char *cmol_version(void);
size_t cmol_arena_estimate(const char *gguf_path, const cmol_config_t *cfg);

int cmol_format_chatml(const char *system, const char *user,
                        char *buf, size_t buf_cap);
int cmol_format_chatml_turn(const char *user, char *buf, size_t buf_cap);

#ifdef __cplusplus
}
#endif

#endif /* CMOL_H */
