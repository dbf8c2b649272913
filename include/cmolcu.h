/*
 * cmolcu.h — the C ABI of the B200 kernel layer of libcmol-b200.
 *
 * This is the inner seam between the host C/C++ runtime (public API in
 * cmol.h) and the sm_100a kernels.  It replaces two reference interfaces:
 *
 *   - the quantised matmul function pointer cmol_matmul_fn_t
 *     (src/cmol_internal.h:175-187 of nvlass/libcmol), whose only
 *     implementations are the CPU kernels of src/quant.c:334-566;
 *   - the per-token forward pass cmol_model_forward (src/model.h:21-24),
 *     replaced by the batched decode step of the engine (cmol_cuda.h).
 *
 * Conventions: plain pointers and sizes only; functions returning int give
 * 0 on success and -1 on failure, with a message in cmolcu_last_error()
 * (per thread).  No C++ exception crosses this boundary.  A `stream`
 * argument is a cudaStream_t passed as void* (NULL = legacy default stream).
 */
#ifndef CMOLCU_H
#define CMOLCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type tags accepted by the kernels (GGUF numbering). */
#define CMOLCU_F32  0
#define CMOLCU_F16  1
#define CMOLCU_Q4_0 2
#define CMOLCU_Q5_0 6
#define CMOLCU_Q8_0 8
#define CMOLCU_Q4_K 12
#define CMOLCU_Q6_K 14

/* Message of the last failure on the calling thread ("" if none). */
const char *cmolcu_last_error(void);

/* Number of CUDA devices visible to the process. */
int cmolcu_device_count(void);

/* Device fault word of the kernels launched through this header on
 * `device`: 0 = no fault; otherwise a pipeline wait gave up (1: a consumer
 * waited too long for data, 2: a producer waited too long for a free
 * stage) and the affected outputs are invalid.  Waits in these kernels are
 * bounded, so such a fault is reported here instead of hanging the GPU.
 * `clear` resets the word. */
int cmolcu_fault_status(int device, unsigned int *code, int clear);

/* ---- quantised weights ---------------------------------------------------
 * A weight is a [rows x k] matrix given as GGUF blocks (row-major, rows of
 * (k / block_values) packed blocks, exactly the layout `a` has in
 * cmol_matmul_fn_t).  Upload repacks it on the device into 16-byte aligned
 * planes; the values are unchanged. */
typedef struct cmolcu_weight cmolcu_weight_t;

int    cmolcu_weight_upload(int device, const void *gguf_rows, int dtype, int rows, int k,
                            cmolcu_weight_t **out);
/* Same, from GGUF rows already in device memory (on `device`). */
int    cmolcu_weight_upload_dev(int device, const void *gguf_rows_dev, int dtype, int rows, int k,
                                cmolcu_weight_t **out);
void   cmolcu_weight_free(cmolcu_weight_t *w);
size_t cmolcu_weight_bytes(const cmolcu_weight_t *w);   /* GGUF bytes = bytes one pass reads */

/* ---- dequant-dot GEMV on device buffers ----------------------------------
 *   y(c, r) = sum_k deq(W[r, k]) * xn(c, k)          c < n
 *   x(c, i) = x[c * x_ld + i * x_inc],  y(c, r) = y[c * y_ld + r * y_inc]
 *   xn = x, or w[i] * (x[i] * 1/sqrt(mean(x^2) + eps)) when norm_w != NULL
 * x_inc = n, x_ld = 1, y_ld = 1, y_inc = n is the cmol_matmul_fn_t layout
 * (b[k*n+ni], out[mi*n+ni]).  Replaces src/quant.c:334-566. */
int cmolcu_gemv(const cmolcu_weight_t *w,
                const float *x, long long x_ld, int x_inc, int n,
                const float *norm_w, float eps,
                float *y, long long y_ld, int y_inc, void *stream);

/* ---- batched matmul on the tensor cores ------------------------------------
 * y(c, r) = sum_k deq(W[r, k]) * xn(c, k) for c < n <= 256 columns, device
 * buffers x [n][k] and y [n][rows], xn as in cmolcu_gemv.  Weights are
 * dequantised to f16 and activations rounded to f16, products accumulate in
 * f32 (tcgen05): results differ from cmolcu_gemv by about 2^-11 relative
 * per term.  Q4_K, Q8_0, Q4_0 and Q5_0 only; k a multiple of 64.  Replaces
 * the n > 1 use of src/quant.c:334-566 (which re-dequantises per column). */
int cmolcu_matmul_batched(const cmolcu_weight_t *w, const float *x, int n, const float *norm_w, float eps,
                          float *y, void *stream);

/* Microbenchmark of the tensor-core path: `iters` back-to-back
 * cmolcu_matmul_batched products (rotating over the nw weights of one
 * shape, n <= 256 columns, x [n][k], y [n][rows] on the device) captured in
 * one CUDA graph and replayed `reps` times; device time per product. */
int cmolcu_matmul_batched_bench(cmolcu_weight_t *const *ws, int nw, const float *x, int n, float *y,
                                int iters, int reps, float *ms_per_matmul);

/* Microbenchmark: `iters` back-to-back GEMVs (rotating over the nw weights,
 * all of one shape, n = 1..16 columns (one launch per 2, as the engine runs
 * them), x [n][k], y [n][rows] on the
 * device), captured once in a CUDA graph with programmatic dependent launch
 * and replayed `reps` times.  *ms_per_gemv is device time per GEMV measured
 * with CUDA events on the replay stream. */
int cmolcu_gemv_bench(cmolcu_weight_t *const *ws, int nw, const float *x, int n, float *y,
                      int iters, int reps, float *ms_per_gemv);

/* ---- the matmul seam on host buffers -------------------------------------
 * Exactly the signature and semantics of cmol_matmul_fn_t
 * (src/cmol_internal.h:175-182): out[m*n] = A[m*k] . B[k*n] with A in GGUF
 * blocks of `dtype` and host pointers throughout.  Uploads, runs on the
 * current device and copies back.  On failure (or an unknown dtype) `out` is
 * left untouched, as the reference's kernels do (src/quant.c:337-338);
 * cmolcu_last_error() says why. */
void cmolcu_matmul(float *out, const void *a, const float *b,
                   int m, int k, int n, int dtype);

/* ---- the matmul seam without device allocation -----------------------------
 * No counterpart in the reference (its matmul never touches a device).
 * cmolcu_matmul, same signature and results, but it allocates no device
 * memory: no cudaMalloc/cudaFree or other allocating call.  It is for callers
 * that cannot allocate: code running beside a live decode engine (cudaFree
 * waits for the whole device and would stall its streams) or under a memory
 * pool that already holds the free memory.  All working memory lives in one
 * static device array of CMOLCU_NOALLOC_SCRATCH_BYTES per device:
 *   256 + up256(m * row_bytes(k)) + up256(repacked planes of A)
 *       + up256(4*k*n) + up256(4*m*n)       must be <= the limit
 * (up256 = round up to 256; e.g. 11008 x 2048 Q8_0 fits up to n = 367).
 * Larger requests are rejected: out untouched, cmolcu_last_error() says so.
 * cmolcu_last_error() is "" after a call that succeeded.
 * The first call on each device looks up the scratch address and sets the
 * GEMV's shared-memory attribute; make it before any stream capture.  The
 * address is kept for the life of the process: do not call this again on a
 * device after cudaDeviceReset.  The array is part of every CUDA context
 * that loads libcmol.so, the decode engine's included. 
 * Calls on one device share the scratch: overlapping calls (two threads at
 * once) race and must be serialised by the caller. */
#define CMOLCU_NOALLOC_SCRATCH_BYTES (64u << 20)
void cmolcu_matmul_noalloc(float *out, const void *a, const float *b,
                           int m, int k, int n, int dtype);

/* ---- host-only tokenizer -------------------------------------------------
 * The vocabulary of a GGUF file without loading weights or using a GPU:
 * the same encoder and decoder cmol_encode / cmol_decode_token use
 * (replaces src/tokenizer.c:359-571 of the reference; encode uses the
 * file's add_bos flag).  Return codes are cmol_err_t values. */
typedef struct cmolcu_tokenizer cmolcu_tokenizer_t;
int         cmolcu_tokenizer_open(const char *gguf_path, cmolcu_tokenizer_t **out);
int         cmolcu_tokenizer_encode(const cmolcu_tokenizer_t *t, const char *text, int32_t *out, int cap);
const char *cmolcu_tokenizer_decode(const cmolcu_tokenizer_t *t, int32_t id);
void        cmolcu_tokenizer_free(cmolcu_tokenizer_t *t);

#ifdef __cplusplus
}
#endif
#endif /* CMOLCU_H */
