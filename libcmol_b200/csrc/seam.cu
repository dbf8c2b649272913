// seam.cu — the C ABI of cmolcu.h (weights, GEMV, host matmul seam).
#include "../../include/cmolcu.h"
#include "gemm_tc.cuh"
#include "gemv_launch.cuh"

#include <stdarg.h>
#include <string.h>

#include <algorithm>
#include <string>

static thread_local char g_err[512];

extern "C" void cmolcu_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

extern "C" const char *cmolcu_last_error(void) { return g_err; }

// One fault word per device for kernels launched through this seam.
static unsigned int *g_fault[64];

unsigned int *cmolcu_fault_word(int device) {
    if (device < 0 || device >= 64) return nullptr;
    if (!g_fault[device]) {
        unsigned int *p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned int)) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, sizeof(unsigned int));
        g_fault[device] = p;
    }
    return g_fault[device];
}

extern "C" int cmolcu_fault_status(int device, unsigned int *code, int clear) {
    unsigned int *p = cmolcu_fault_word(device);
    if (!p) { cmolcu_set_error("no fault word for device %d", device); return -1; }
    unsigned int v = 0;
    CUDA_TRY(cudaSetDevice(device));
    CUDA_TRY(cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost));
    if (clear && v) CUDA_TRY(cudaMemset(p, 0, sizeof(unsigned int)));
    if (code) *code = v;
    return 0;
}

extern "C" int cmolcu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

struct cmolcu_weight {
    QWeight w;
    int     device;
    void   *base;       // single allocation holding all planes
};

static bool dtype_ok(int dt) {
    return dt == DT_F32 || dt == DT_F16 || dt == DT_Q4_0 || dt == DT_Q5_0 ||
           dt == DT_Q8_0 || dt == DT_Q4_K || dt == DT_Q6_K;
}

// Allocate the padded planes of a [rows x k] weight on the current device
// (rows rounded up to 32, plane rows to 16 bytes; padding zeroed).
static int weight_alloc(int device, int dtype, int rows, int k, cmolcu_weight_t **out) {
    if (!dtype_ok(dtype)) { cmolcu_set_error("unsupported dtype %d", dtype); return -1; }
    int bv = dt_block_values(dtype);
    if (rows <= 0 || k <= 0 || k % bv != 0 || k % 16 != 0) {
        cmolcu_set_error("bad shape rows=%d k=%d for dtype %d", rows, k, dtype);
        return -1;
    }
    QWeight q = {};
    const size_t tot = qw_layout(q, dtype, rows, k, qw_default_kc(dtype, k));
    void *base = nullptr;
    CUDA_TRY(cudaMalloc(&base, tot));
    CUDA_TRY(cudaMemset(base, 0, tot));
    cmolcu_weight_t *w = new cmolcu_weight_t();
    w->device = device;
    w->base = base;
    for (int i = 0; i < q.nplanes; i++) q.p[i] = (uint8_t *)base + (uintptr_t)q.p[i];
    w->w = q;
    *out = w;
    return 0;
}

static int upload_common(int device, const void *src, bool src_dev, int dtype, int rows, int k,
                         cmolcu_weight_t **out) {
    if (!out || !src) { cmolcu_set_error("NULL argument"); return -1; }
    *out = nullptr;
    CUDA_TRY(cudaSetDevice(device));
    cmolcu_weight_t *w = nullptr;
    if (weight_alloc(device, dtype, rows, k, &w)) return -1;
    const uint8_t *dsrc = (const uint8_t *)src;
    void *tmp = nullptr;
    if (!src_dev) {
        cudaError_t e = cudaMalloc(&tmp, w->w.bytes);
        if (e == cudaSuccess) e = cudaMemcpy(tmp, src, w->w.bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cmolcu_set_error("upload: %s", cudaGetErrorString(e));
            if (tmp) cudaFree(tmp);
            cmolcu_weight_free(w);
            return -1;
        }
        dsrc = (const uint8_t *)tmp;
    }
    cudaError_t e = repack_launch(dsrc, w->w, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        cmolcu_set_error("repack: %s", cudaGetErrorString(e));
        cmolcu_weight_free(w);
        return -1;
    }
    *out = w;
    return 0;
}

extern "C" int cmolcu_weight_upload(int device, const void *gguf_rows, int dtype, int rows, int k,
                                    cmolcu_weight_t **out) {
    return upload_common(device, gguf_rows, false, dtype, rows, k, out);
}

extern "C" int cmolcu_weight_upload_dev(int device, const void *gguf_rows_dev, int dtype, int rows,
                                        int k, cmolcu_weight_t **out) {
    return upload_common(device, gguf_rows_dev, true, dtype, rows, k, out);
}

extern "C" void cmolcu_weight_free(cmolcu_weight_t *w) {
    if (!w) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(w->device);
    cudaFree(w->base);
    cudaSetDevice(cur);
    delete w;
}

extern "C" size_t cmolcu_weight_bytes(const cmolcu_weight_t *w) { return w ? w->w.bytes : 0; }

const QWeight *cmolcu_weight_q(const cmolcu_weight_t *w) { return w ? &w->w : nullptr; }

extern "C" int cmolcu_gemv(const cmolcu_weight_t *w, const float *x, long long x_ld, int x_inc, int n,
                           const float *norm_w, float eps, float *y, long long y_ld, int y_inc,
                           void *stream) {
    if (!w || !x || !y || n <= 0) { cmolcu_set_error("cmolcu_gemv: bad arguments"); return -1; }
    GemvArgs a = {};
    a.w = w->w;
    a.x = x; a.x_ld = x_ld; a.x_inc = x_inc;
    a.norm_w = norm_w; a.eps = eps;
    a.y = y; a.y_ld = y_ld; a.y_inc = y_inc;
    CUDA_TRY(cudaSetDevice(w->device));
    a.fault = cmolcu_fault_word(w->device);
    CUDA_TRY(gemv_launch_cols(a, n, EPI_STORE, (cudaStream_t)stream, false));
    return 0;
}

extern "C" void cmolcu_matmul(float *out, const void *a, const float *b, int m, int k, int n, int dtype) {
    if (!out || !a || !b || m <= 0 || k <= 0 || n <= 0) { cmolcu_set_error("cmolcu_matmul: bad arguments"); return; }
    int dev = 0;
    cudaGetDevice(&dev);
    cmolcu_weight_t *w = nullptr;
    if (cmolcu_weight_upload(dev, a, dtype, m, k, &w)) return;
    float *db = nullptr, *dy = nullptr;
    cudaError_t e = cudaMalloc(&db, (size_t)k * n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&dy, (size_t)m * n * 4);
    if (e == cudaSuccess) e = cudaMemcpy(db, b, (size_t)k * n * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && cmolcu_gemv(w, db, 1, n, n, nullptr, 0.f, dy, 1, n, nullptr) != 0)
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaMemcpy(out, dy, (size_t)m * n * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess && e != cudaErrorUnknown) cmolcu_set_error("cmolcu_matmul: %s", cudaGetErrorString(e));
    cudaFree(db);
    cudaFree(dy);
    cmolcu_weight_free(w);
}

extern "C" int cmolcu_matmul_batched(const cmolcu_weight_t *w, const float *x, int n, const float *norm_w,
                                     float eps, float *y, void *stream) {
    if (!w || !x || !y || n < 1 || n > TC_MAX_N) { cmolcu_set_error("cmolcu_matmul_batched: bad arguments"); return -1; }
    if (!tc_supported(w->w.dtype)) {
        cmolcu_set_error("cmolcu_matmul_batched: dtype %d has no tensor-core path", w->w.dtype);
        return -1;
    }
    CUDA_TRY(cudaSetDevice(w->device));
    size_t xh = 0, pf = 0;
    int rb = 0;
    tc_scratch_need(w->w.rows, w->w.k, n, &xh, &pf, &rb);
    TcScratch sc = {};
    cudaError_t e = cudaMalloc(&sc.xs, xh * 2);
    if (e == cudaSuccess) e = cudaMalloc(&sc.part, std::max<size_t>(pf, 1) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&sc.counters, (size_t)rb * 4);
    if (e == cudaSuccess) e = cudaMemset(sc.counters, 0, (size_t)rb * 4);
    sc.part_floats = pf;
    sc.max_row_blocks = rb;
    unsigned int *fw = cmolcu_fault_word(w->device);
    if (e == cudaSuccess) {
        GemvArgs a = {};
        a.w = w->w;
        a.x = x; a.x_ld = w->w.k; a.x_inc = 1;
        a.norm_w = norm_w; a.eps = eps;
        a.y = y; a.y_ld = w->w.rows; a.y_inc = 1;
        a.fault = fw;
        e = tc_matmul(a, n, EPI_STORE, sc, (cudaStream_t)stream, false);
        if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    }
    cudaFree(sc.xs);
    cudaFree(sc.part);
    cudaFree(sc.counters);
    if (e != cudaSuccess) { cmolcu_set_error("cmolcu_matmul_batched: %s", cudaGetErrorString(e)); return -1; }
    return 0;
}

// Back-to-back tensor-core matmuls over `nw` distinct weights (one shape),
// n columns, captured once in a CUDA graph (two launches each) and replayed
// `reps` times; *ms_per_matmul from CUDA events on the replay stream.
extern "C" int cmolcu_matmul_batched_bench(cmolcu_weight_t *const *ws, int nw, const float *x, int n, float *y,
                                           int iters, int reps, float *ms_per_matmul) {
    if (!ws || nw <= 0 || !x || !y || n < 1 || n > TC_MAX_N || iters <= 0 || reps <= 0 || !ms_per_matmul) {
        cmolcu_set_error("cmolcu_matmul_batched_bench: bad arguments");
        return -1;
    }
    if (!tc_supported(ws[0]->w.dtype)) { cmolcu_set_error("cmolcu_matmul_batched_bench: dtype has no tensor-core path"); return -1; }
    const int dev = ws[0]->device;
    CUDA_TRY(cudaSetDevice(dev));
    size_t xh = 0, pf = 0;
    int rb = 0;
    tc_scratch_need(ws[0]->w.rows, ws[0]->w.k, n, &xh, &pf, &rb);
    TcScratch sc = {};
    cudaStream_t st = nullptr;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    unsigned int *fw = cmolcu_fault_word(dev);
    cudaError_t err = cudaMalloc(&sc.xs, xh * 2);
    if (err == cudaSuccess) err = cudaMalloc(&sc.part, std::max<size_t>(pf, 1) * 4);
    if (err == cudaSuccess) err = cudaMalloc(&sc.counters, (size_t)rb * 4);
    if (err == cudaSuccess) err = cudaMemset(sc.counters, 0, (size_t)rb * 4);
    sc.part_floats = pf;
    sc.max_row_blocks = rb;
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    auto launch_all = [&]() -> cudaError_t {
        for (int i = 0; i < iters; i++) {
            const QWeight &q = ws[i % nw]->w;
            GemvArgs a = {};
            a.w = q;
            a.x = x; a.x_ld = q.k; a.x_inc = 1;
            a.y = y; a.y_ld = q.rows; a.y_inc = 1;
            a.fault = fw;
            cudaError_t e = tc_matmul(a, n, EPI_STORE, sc, st, true);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    };
    if (err == cudaSuccess) err = launch_all();    // eager pass: kernel attributes, warm-up
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err == cudaSuccess) err = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (err == cudaSuccess) {
        cudaError_t re = launch_all();
        err = cudaStreamEndCapture(st, &g);
        if (re != cudaSuccess) err = re;
    }
    if (err == cudaSuccess) err = cudaGraphInstantiate(&ge, g, 0);
    if (err == cudaSuccess) err = cudaEventCreate(&e0);
    if (err == cudaSuccess) err = cudaEventCreate(&e1);
    if (err == cudaSuccess) err = cudaGraphLaunch(ge, st);
    if (err == cudaSuccess) err = cudaEventRecord(e0, st);
    for (int r = 0; err == cudaSuccess && r < reps; r++) err = cudaGraphLaunch(ge, st);
    if (err == cudaSuccess) err = cudaEventRecord(e1, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    float ms = 0.f;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (st) cudaStreamDestroy(st);
    cudaFree(sc.xs);
    cudaFree(sc.part);
    cudaFree(sc.counters);
    if (err != cudaSuccess) { cmolcu_set_error("cmolcu_matmul_batched_bench: %s", cudaGetErrorString(err)); return -1; }
    *ms_per_matmul = ms / (float)(iters * reps);
    return 0;
}

// Back-to-back GEMVs over `nw` distinct weights (all the same shape), captured
// in one CUDA graph with programmatic dependent launch between them, replayed
// `reps` times; *ms_per_gemv = device time per GEMV (CUDA events).  n <= 16
// columns, launched as the engine does (one launch per 2 columns).
extern "C" int cmolcu_gemv_bench(cmolcu_weight_t *const *ws, int nw, const float *x, int n, float *y,
                                 int iters, int reps, float *ms_per_gemv) {
    if (!ws || nw <= 0 || !x || !y || n < 1 || n > 16 || iters <= 0 || reps <= 0 || !ms_per_gemv) {
        cmolcu_set_error("cmolcu_gemv_bench: bad arguments");
        return -1;
    }
    const int dev = ws[0]->device;
    CUDA_TRY(cudaSetDevice(dev));
    cudaStream_t st = nullptr;
    CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    unsigned int *fw = cmolcu_fault_word(dev);   // allocate before capturing
    auto launch_all = [&]() -> cudaError_t {
        for (int i = 0; i < iters; i++) {
            const QWeight &q = ws[i % nw]->w;
            GemvArgs a = {};
            a.w = q;
            a.x = x; a.x_ld = q.k; a.x_inc = 1; a.ncol = n;
            a.y = y; a.y_ld = q.rows; a.y_inc = 1;
            a.fault = fw;
            cudaError_t e = gemv_launch_cols(a, n, EPI_STORE, st, true);   // the engine's column loop
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    };
    cudaError_t err = launch_all();              // eager pass: kernel attributes, warm-up
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err == cudaSuccess) err = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (err == cudaSuccess) err = launch_all();
    cudaError_t e2 = cudaStreamEndCapture(st, &g);
    if (err == cudaSuccess) err = e2;
    if (err == cudaSuccess) err = cudaGraphInstantiate(&ge, g, 0);
    if (err == cudaSuccess) err = cudaEventCreate(&e0);
    if (err == cudaSuccess) err = cudaEventCreate(&e1);
    if (err == cudaSuccess) err = cudaGraphLaunch(ge, st);          // warm-up
    if (err == cudaSuccess) err = cudaEventRecord(e0, st);
    for (int r = 0; err == cudaSuccess && r < reps; r++) err = cudaGraphLaunch(ge, st);
    if (err == cudaSuccess) err = cudaEventRecord(e1, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    float ms = 0.f;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaStreamDestroy(st);
    if (err != cudaSuccess) { cmolcu_set_error("cmolcu_gemv_bench: %s", cudaGetErrorString(err)); return -1; }
    *ms_per_gemv = ms / (float)(iters * reps);
    return 0;
}
