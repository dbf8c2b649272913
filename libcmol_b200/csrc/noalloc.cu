// noalloc.cu — cmolcu_matmul_noalloc: the host matmul seam without any
// device memory allocation.
//
// cmolcu_matmul allocates device buffers on every call (the repacked weight,
// the GGUF rows, b, out) and frees them again.  cudaFree waits for the whole
// device, so a caller that runs next to a live decode engine stalls every
// stream on the GPU each time; a caller whose device memory is already
// claimed by a pool (a framework's caching allocator, a KV pool sized to the
// free memory) may see the allocation fail outright.  This variant keeps all
// of its working memory in one statically sized device array instead, so it
// never calls cudaMalloc, cudaFree or anything else that allocates.
//
// Scratch layout (each part starts on a 256-byte boundary):
//   [fault word][GGUF rows of A][repacked planes of A][b: k*n floats][out: m*n floats]
// A request whose parts do not fit in CMOLCU_NOALLOC_SCRATCH_BYTES is
// rejected before any device work.
//
// What must start at zero: the fault word and the padding of the repacked
// planes.  Both are cleared with cudaMemsetAsync at the start of every call;
// nothing else is read before it is written.
#include "../../include/cmolcu.h"
#include "gemv_launch.cuh"

#include <mutex>

static __device__ __align__(256) unsigned char g_noalloc_scratch[CMOLCU_NOALLOC_SCRATCH_BYTES];

// Address of g_noalloc_scratch on each device, resolved once per device with
// that device current (the host never passes the symbol itself to a kernel).
// The cache lives as long as the process: after a cudaDeviceReset the module
// may be loaded at another address, so a process that resets a device must
// not call this entry point on it again.
static unsigned char *g_scratch_ptr[64];
static std::mutex g_scratch_mu;

static unsigned char *scratch_for(int dev) {
    if (dev < 0 || dev >= 64) {
        cmolcu_set_error("cmolcu_matmul_noalloc: device %d is above the 64-device table", dev);
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cmolcu_set_error("cmolcu_matmul_noalloc: scratch address on device %d: %s", dev,
                             cudaGetErrorString(e));
            return nullptr;
        }
        g_scratch_ptr[dev] = (unsigned char *)p;
    }
    return g_scratch_ptr[dev];
}

static size_t up256(size_t b) { return (b + 255) & ~(size_t)255; }

extern "C" void cmolcu_matmul_noalloc(float *out, const void *a, const float *b, int m, int k, int n,
                                      int dtype) {
    cmolcu_set_error("%s", "");
    if (!out || !a || !b || m <= 0 || k <= 0 || n <= 0) {
        cmolcu_set_error("cmolcu_matmul_noalloc: bad arguments");
        return;
    }
    const int bv = dt_block_values(dtype);
    if (bv <= 0 || k % bv != 0 || k % 16 != 0) {
        cmolcu_set_error("cmolcu_matmul_noalloc: bad shape k=%d for dtype %d", k, dtype);
        return;
    }
    if (k > CMOLCU_GEMV_MAX_K) {
        cmolcu_set_error("cmolcu_matmul_noalloc: k=%d above %d", k, CMOLCU_GEMV_MAX_K);
        return;
    }
    QWeight q = {};
    const size_t planes = qw_layout(q, dtype, m, k, qw_default_kc(dtype, k));
    const size_t raw = (size_t)m * dt_row_bytes(k, dtype);
    const size_t o_raw = 256;
    const size_t o_planes = o_raw + up256(raw);
    const size_t o_b = o_planes + up256(planes);
    const size_t o_y = o_b + up256((size_t)k * n * 4);
    const size_t need = o_y + up256((size_t)m * n * 4);
    if (need > (size_t)CMOLCU_NOALLOC_SCRATCH_BYTES) {
        cmolcu_set_error("cmolcu_matmul_noalloc: m=%d k=%d n=%d dtype %d needs %zu bytes of scratch, "
                         "above the %zu-byte limit", m, k, n, dtype, need,
                         (size_t)CMOLCU_NOALLOC_SCRATCH_BYTES);
        return;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cmolcu_set_error("cmolcu_matmul_noalloc: no device"); return; }
    unsigned char *s = scratch_for(dev);
    if (!s) return;

    for (int i = 0; i < q.nplanes; i++) q.p[i] = s + o_planes + (uintptr_t)q.p[i];
    unsigned int *fault = reinterpret_cast<unsigned int *>(s);
    float *db = reinterpret_cast<float *>(s + o_b);
    float *dy = reinterpret_cast<float *>(s + o_y);

    cudaStream_t st = nullptr;   // the legacy stream, as cmolcu_matmul
    cudaError_t e = cudaMemsetAsync(s, 0, 256, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s + o_planes, 0, planes, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s + o_raw, a, raw, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(db, b, (size_t)k * n * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = repack_launch(s + o_raw, q, st);
    if (e == cudaSuccess) {
        GemvArgs ga = {};
        ga.w = q;
        ga.x = db; ga.x_ld = 1; ga.x_inc = n;
        ga.y = dy; ga.y_ld = 1; ga.y_inc = n;
        ga.fault = fault;
        e = gemv_launch_cols(ga, n, EPI_STORE, st, false);
    }
    unsigned int code = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&code, fault, sizeof code, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { cmolcu_set_error("cmolcu_matmul_noalloc: %s", cudaGetErrorString(e)); return; }
    if (code) { cmolcu_set_error("cmolcu_matmul_noalloc: device fault %u", code); return; }
    e = cudaMemcpy(out, dy, (size_t)m * n * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) cmolcu_set_error("cmolcu_matmul_noalloc: %s", cudaGetErrorString(e));
}
