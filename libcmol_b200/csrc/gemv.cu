// gemv.cu — template instances, launch planning and weight repacking.
#include "gemv_launch.cuh"

#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>

// ---------------------------------------------------------------------------
// Repack: one thread per GGUF block, bytes copied into the padded planes
// described in qweight.cuh.  Runs once per tensor at load time.
// ---------------------------------------------------------------------------
__global__ void k_repack(const uint8_t *src, QWeight w) {
    const int dt = w.dtype;
    const int bv = dt_block_values(dt), bb = dt_block_bytes(dt);
    const long long nb = w.k / bv;
    const int bpc = w.kc / bv;            // blocks per K-chunk
    const long long total = (long long)w.rows * nb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / nb, blk = i % nb;
        const int j = (int)(blk / bpc), lb = (int)(blk % bpc);
        const uint8_t *s = src + row * nb * bb + blk * bb;
        uint8_t *p0 = qw_row(w, 0, j, row);
        uint8_t *p1 = w.nplanes > 1 ? qw_row(w, 1, j, row) : nullptr;
        uint8_t *p2 = w.nplanes > 2 ? qw_row(w, 2, j, row) : nullptr;
        uint8_t *p3 = w.nplanes > 3 ? qw_row(w, 3, j, row) : nullptr;
        switch (dt) {
        case DT_Q8_0:
            p1[lb * 2] = s[0]; p1[lb * 2 + 1] = s[1];
            for (int t = 0; t < 32; t++) p0[lb * 32 + t] = s[2 + t];
            break;
        case DT_Q4_0:
            p1[lb * 2] = s[0]; p1[lb * 2 + 1] = s[1];
            for (int t = 0; t < 16; t++) p0[lb * 16 + t] = s[2 + t];
            break;
        case DT_Q5_0:
            p1[lb * 2] = s[0]; p1[lb * 2 + 1] = s[1];
            for (int t = 0; t < 4; t++) p2[lb * 4 + t] = s[2 + t];
            for (int t = 0; t < 16; t++) p0[lb * 16 + t] = s[6 + t];
            break;
        case DT_Q4_K:
            for (int t = 0; t < 16; t++) p1[lb * 16 + t] = s[t];
            for (int t = 0; t < 128; t++) p0[lb * 128 + t] = s[16 + t];
            break;
        case DT_Q6_K:
            for (int t = 0; t < 128; t++) p0[lb * 128 + t] = s[t];
            for (int t = 0; t < 64; t++) p1[lb * 64 + t] = s[128 + t];
            for (int t = 0; t < 16; t++) p2[lb * 16 + t] = s[192 + t];
            p3[lb * 2] = s[208]; p3[lb * 2 + 1] = s[209];
            break;
        case DT_F16:
            for (int t = 0; t < 2; t++) p0[lb * 2 + t] = s[t];
            break;
        case DT_F32:
            for (int t = 0; t < 4; t++) p0[lb * 4 + t] = s[t];
            break;
        default: break;
        }
    }
}

cudaError_t repack_launch(const uint8_t *src, QWeight w, cudaStream_t st) {
    long long total = (long long)w.rows * (w.k / dt_block_values(w.dtype));
    int blocks = (int)std::min<long long>((total + 255) / 256, 65535LL * 4);
    k_repack<<<blocks, 256, 0, st>>>(src, w);
    return cudaGetLastError();
}

int device_sm_count() {
    static int cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// ---------------------------------------------------------------------------
// Dispatch
// ---------------------------------------------------------------------------
typedef void (*gemv_kernel_t)(GemvArgs);

template <int DT, int NC, int R, int CW>
static gemv_kernel_t pick_epi(int epi) {
    switch (epi) {
    case EPI_STORE:  return k_gemv<DT, NC, R, EPI_STORE, CW>;
    case EPI_RESID:  return k_gemv<DT, NC, R, EPI_RESID, CW>;
    case EPI_SWIGLU: return k_gemv<DT, NC, R, EPI_SWIGLU, CW>;
    case EPI_QKV:    return k_gemv<DT, NC, R, EPI_QKV, CW>;
    default: return nullptr;
    }
}

template <int DT>
static gemv_kernel_t pick_dt(int nc, int r, int epi, int cw) {
    if (r != 4) return nullptr;
    if (cw == GEMV_CWARPS_WIDE) return nc == 1 ? pick_epi<DT, 1, 4, GEMV_CWARPS_WIDE>(epi) : pick_epi<DT, 2, 4, GEMV_CWARPS_WIDE>(epi);
    return nc == 1 ? pick_epi<DT, 1, 4, GEMV_CWARPS>(epi) : pick_epi<DT, 2, 4, GEMV_CWARPS>(epi);
}

static gemv_kernel_t pick(int dt, int nc, int r, int epi, int cw) {
    switch (dt) {
    case DT_Q8_0: return pick_dt<DT_Q8_0>(nc, r, epi, cw);
    case DT_Q4_0: return pick_dt<DT_Q4_0>(nc, r, epi, cw);
    case DT_Q5_0: return pick_dt<DT_Q5_0>(nc, r, epi, cw);
    case DT_Q4_K: return pick_dt<DT_Q4_K>(nc, r, epi, cw);
    case DT_Q6_K: return pick_dt<DT_Q6_K>(nc, r, epi, cw);
    case DT_F16:  return pick_dt<DT_F16>(nc, r, epi, cw);
    case DT_F32:  return pick_dt<DT_F32>(nc, r, epi, cw);
    default: return nullptr;
    }
}

static std::mutex g_attr_mu;

// Raise the kernel's dynamic shared-memory limit to what the device allows
// next to its static shared memory; returns that limit (bytes).
static size_t ensure_smem_attr(gemv_kernel_t k) {
    static gemv_kernel_t done[1024];
    static int dev_done[1024];
    static size_t lim_done[1024];
    static int n = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_attr_mu);
    for (int i = 0; i < n; i++)
        if (done[i] == k && dev_done[i] == dev) return lim_done[i];
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa = {};
    cudaFuncGetAttributes(&fa, k);
    size_t lim = (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim) != cudaSuccess) {
        cudaGetLastError();   // do not leave a sticky error behind
        lim = 48 * 1024;
    }
    if (n < 1024) { done[n] = k; dev_done[n] = dev; lim_done[n] = lim; n++; }
    return lim;
}

static void fmt_of(int dt, int &vpc, int &cr) {
    vpc = (dt == DT_Q8_0 || dt == DT_F16 || dt == DT_F32) ? 16 : 32;
    cr = vpc == 16 ? 1 : 2;
}

// Choose rows per warp, rows per CTA, K-chunk and pipeline depth for one
// launch.  Every CTA gets one contiguous range of rows (a multiple of R), so
// the work of an SM is balanced to a few rows.  Small matrices (the decode
// step's) use two CTAs per SM of up to ~100 KB of shared memory each, so the
// next kernel of the step can start streaming while this one drains.  Large
// matrices use one CTA per SM with up to ~216 KB, so an SM's whole share (or
// most of it) is in flight at once.
// CMOLCU_GEMV_PLAN=<kb>:<ctas per SM> (measurements) forces one budget
// and grid for every launch, e.g. 100:1 (the narrow variant, one CTA per SM,
// so that the next kernel's CTAs fit beside this one's).
static void gemv_forced_plan(int &kb, int &per_sm) {
    static int fkb = -1, fps = 0;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *v = getenv("CMOLCU_GEMV_PLAN");
        int a = 0, b = 0;
        if (v && sscanf(v, "%d:%d", &a, &b) == 2 && (a == 100 || a == 216) && b >= 1 && b <= 2) {
            fkb = a;
            fps = b;
        }
    });
    kb = fkb;
    per_sm = fps;
}

bool gemv_plan(const QWeight &w, int nc, PipeCfg &pc, int &R, int &grid) {
    const int sms = device_sm_count();
    R = 4;
    int vpc, cr;
    fmt_of(w.dtype, vpc, cr);
    const size_t xb = gemv_x_bytes(nc, w.k, vpc, cr);
    const bool large = w.bytes >= (size_t)4 << 20;
    int forced_kb = -1, forced_per_sm = 0;
    gemv_forced_plan(forced_kb, forced_per_sm);
    const int order[3][2] = {{100, 216}, {216, 100}, {forced_kb, forced_kb == 100 ? 216 : 100}};
    for (int budget_kb : order[forced_kb > 0 ? 2 : large ? 1 : 0]) {
        // one CTA per SM gets the wide variant (15 consumer warps)
        const int cw = budget_kb <= 100 ? GEMV_CWARPS : GEMV_CWARPS_WIDE;
        const int tr = cw * R;
        int off = 0;
        for (int p = 0; p < 4; p++) {
            pc.po[p] = off;
            off += p < w.nplanes ? tr * w.cs[p] : 0;
        }
        pc.sb = off;
        pc.cw = cw;
        const long long avail = (long long)budget_kb * 1024 - (long long)xb - 2 * GEMV_MAX_STAGES * 8;
        if (avail < 2LL * pc.sb) continue;
        const int ctas = sms * (forced_per_sm > 0 && budget_kb == forced_kb ? forced_per_sm : budget_kb <= 100 ? 2 : 1);
        int rpc = (w.rows + ctas - 1) / ctas;
        rpc = (rpc + R - 1) / R * R;
        pc.rows_per_cta = rpc;
        grid = (w.rows + rpc - 1) / rpc;
        const int per_cta = ((rpc + tr - 1) / tr) * w.nkc;
        const int nst = (int)std::min<long long>(GEMV_MAX_STAGES, avail / pc.sb);
        pc.nstage = std::max(1, std::min(nst, per_cta));
        return true;
    }
    return false;
}

cudaError_t gemv_launch(const GemvArgs &a0, int epi, cudaStream_t st, bool pdl) {
    GemvArgs a = a0;
    if (a.ncol < 1 || a.ncol > 2) return cudaErrorInvalidValue;
    if (a.w.k <= 0 || a.w.k > CMOLCU_GEMV_MAX_K || a.w.k % dt_block_values(a.w.dtype) != 0 ||
        a.w.k % 16 != 0)
        return cudaErrorInvalidValue;
    if (a.x_inc == 1 && (((uintptr_t)a.x & 15) || (a.ncol > 1 && (a.x_ld & 3)))) return cudaErrorMisalignedAddress;
    if (a.norm_w && ((uintptr_t)a.norm_w & 15)) return cudaErrorMisalignedAddress;
    int R = 4, grid = 1;
    if (!gemv_plan(a.w, a.ncol, a.pc, R, grid)) return cudaErrorInvalidValue;
    gemv_kernel_t k = pick(a.w.dtype, a.ncol, R, epi, a.pc.cw);
    if (!k) return cudaErrorInvalidValue;
    const size_t lim = ensure_smem_attr(k);
    int vpc, cr;
    fmt_of(a.w.dtype, vpc, cr);
    size_t smem = gemv_smem_total(a.ncol, a.w.k, vpc, cr, a.pc);
    if (smem > lim) return cudaErrorInvalidConfiguration;
    return launch_k(k, dim3(grid), dim3((a.pc.cw + 1) * 32), smem, st, pdl, a);
}

cudaError_t gemv_launch_cols(GemvArgs a, int ncol, int epi, cudaStream_t st, bool pdl) {
    for (int c0 = 0; c0 < ncol; c0 += 2) {
        GemvArgs b = a;
        b.ncol = std::min(2, ncol - c0);
        b.x = a.x + (long long)c0 * a.x_ld;
        b.y = a.y + (long long)c0 * a.y_ld;
        if (epi == EPI_QKV) {
            b.qkv.pos = a.qkv.pos + c0;
            if (a.qkv.slot) b.qkv.slot = a.qkv.slot + c0;
            else b.qkv.page_table = a.qkv.page_table + (long long)c0 * a.qkv.max_pages;
        }
        cudaError_t e = gemv_launch(b, epi, st, pdl);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
