// decode_step.cu — the persistent decode-step kernel (see decode_step.cuh).
#include "attention_item.cuh"
#include "decode_step.cuh"
#include "gemv_launch.cuh"

#include <stdio.h>
#include <stdlib.h>

#include <algorithm>

#define DS_CWARPS 8
#define DS_CTHREADS (DS_CWARPS * 32)
#define DS_THREADS (DS_CTHREADS + 32)
#define DS_R 4                      // rows per warp group
#define DS_TR (DS_CWARPS * DS_R)    // rows per ring slot
#define DS_SYNC_LIMIT (1u << 21)    // polls of the barrier counter before giving up

static_assert(DS_CTHREADS == ATTN_THREADS, "the attention item runs on the consumer warps");

#define DS_MAX_HALF_HD 64          // d_head / 2 for d_head <= 128

struct DsShared {
    AttnShared at;
    float      red_ss[DS_CWARPS][DS_MAX_NC];
    float      inv_rms[DS_MAX_NC];
    float      kred[2][DS_CWARPS][DS_R * DS_MAX_NC];
    int        flag;
    int        abort;                // consumers left early: the producer drains and leaves
    // per-step constants, loaded once at the start of the step
    int        pos[DS_MAX_NC];       // position of each column (< 0: inactive)
    int        cur_page[DS_MAX_NC];  // page holding `pos`
    float2     cs[DS_MAX_NC][DS_MAX_HALF_HD];   // RoPE (cos, sin) at `pos`
};

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned int atom_add_release_gpu(unsigned int *p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Grid barrier of the consumer warps (the producer never takes part).
// Returns false, on every consumer thread, when the wait ran out or any CTA
// has recorded a fault: the step is abandoned.
__device__ __forceinline__ bool ds_grid_sync(unsigned int *count, unsigned int target, unsigned int *fault,
                                             int tid, DsShared &sh) {
    named_bar_sync(1, DS_CTHREADS);
    if (tid == 0) {
        int ok = 1;
        __threadfence();
        const unsigned int old = atom_add_release_gpu(count, 1u);
        if (old + 1u < target) {
            for (uint32_t it = 0;; it++) {
                if (ld_acquire_gpu(count) >= target) break;
                if ((it & 63u) == 63u && *(volatile unsigned int *)fault) { ok = 0; break; }
                if (it >= DS_SYNC_LIMIT) { atomicExch(fault, FAULT_GRID_SYNC); ok = 0; break; }
            }
        }
        __threadfence();
        if (ok && *(volatile unsigned int *)fault) ok = 0;
        sh.flag = ok;
        if (!ok) sh.abort = 1;
    }
    named_bar_sync(1, DS_CTHREADS);
    return sh.flag != 0;
}

__device__ __forceinline__ void ds_rows(const GemvArgs &g, int &rb, int &re) {
    rb = min(g.w.rows, (int)blockIdx.x * g.pc.rows_per_cta);
    re = min(g.w.rows, rb + g.pc.rows_per_cta);
}

// Bounded wait that also gives up when the consumers have left.
__device__ __forceinline__ bool ds_wait_empty(uint64_t *bar, uint32_t parity, unsigned int *fault,
                                              const DsShared &sh) {
    for (uint32_t i = 0; i < CMOLCU_SPIN_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *(volatile const int *)&sh.abort) return false;
    }
    atomicExch(fault, FAULT_GEMV_EMPTY);
    return false;
}

// ---------------------------------------------------------------------------
// Producer warp: every GEMV phase's rows of this CTA, tile by tile, K-chunk
// by K-chunk, one bulk copy per plane into the next ring slot.
// ---------------------------------------------------------------------------
__device__ void ds_producer(const DsArgs &a, uint8_t *ring, uint64_t *full, uint64_t *empty, DsShared &sh,
                            int lane) {
    uint32_t seq = 0;
    bool stop = false;
    for (int p = 0; p < a.n_phases && !stop; p++) {
        const DsPhase *ph = a.phases + p;
        if (ph->kind != DS_GEMV) continue;
        const QWeight w = ph->g.w;
        int po[4];
#pragma unroll
        for (int q = 0; q < 4; q++) po[q] = ph->g.pc.po[q];
        int rb, re;
        ds_rows(ph->g, rb, re);
        const int ntile = (re - rb + DS_TR - 1) / DS_TR;
        if (ph->g.norm_w && ntile > 0) {
            // the RMSNorm gains of the phase travel through the ring too
            const uint32_t s = seq % (uint32_t)a.nslot, n = seq / (uint32_t)a.nslot;
            if (n > 0 && !ds_wait_empty(&empty[s], (n - 1) & 1, a.fault, sh)) { stop = true; break; }
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(w.k * 4));
                bulk_g2s(ring + (size_t)s * a.slot_bytes, ph->g.norm_w, (uint32_t)(w.k * 4), &full[s]);
            }
            __syncwarp();
            seq++;
        }
        for (int ti = 0; ti < ntile && !stop; ti++) {
            const int r0 = rb + ti * DS_TR, nrow = min(DS_TR, re - r0);
            for (int j = 0; j < w.nkc; j++) {
                const uint32_t s = seq % (uint32_t)a.nslot, n = seq / (uint32_t)a.nslot;
                if (n > 0 && !ds_wait_empty(&empty[s], (n - 1) & 1, a.fault, sh)) { stop = true; break; }
                if (lane == 0) {
                    int bytes = 0;
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (q < w.nplanes) bytes += nrow * qw_stride(w, q, j);
                    mbar_arrive_expect_tx(&full[s], (uint32_t)bytes);
                    uint8_t *dst = ring + (size_t)s * a.slot_bytes;
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (q < w.nplanes)
                            bulk_g2s(dst + po[q], qw_row(w, q, j, r0), (uint32_t)(nrow * qw_stride(w, q, j)),
                                     &full[s]);
                }
                __syncwarp();
                seq++;
            }
        }
    }
    if (stop) {
        // copies still in flight land before the CTA's shared memory goes away
        const uint32_t first = seq > (uint32_t)a.nslot ? seq - (uint32_t)a.nslot : 0u;
        for (uint32_t q = first; q < seq; q++) mbar_wait(&full[q % a.nslot], (q / a.nslot) & 1, nullptr, 0);
    }
}

// ---------------------------------------------------------------------------
// Consumer side of a GEMV phase.
// ---------------------------------------------------------------------------

// Q/K/V epilogue with the step's constants from shared memory (position,
// current page, RoPE row): the arithmetic of gemv_epilogue<EPI_QKV>.
template <int NC>
__device__ __forceinline__ void ds_epi_qkv(const GemvArgs &g, const DsShared &sh, int row0, const float *vals,
                                           int lane) {
    if (lane >= (DS_R / 2) * NC) return;
    const EpiQKV &e = g.qkv;
    const int p = lane / NC, col = lane % NC;
    const int row = row0 + 2 * p;
    const int pos = col < g.ncol ? sh.pos[col] : -1;
    if (row + 1 >= g.w.rows || pos < 0) return;
    float v0 = vals[(2 * p) * NC + col], v1 = vals[(2 * p + 1) * NC + col];
    const int D = e.d_model, KVD = e.kv_dim, hd = e.d_head;
    const bool is_v = row >= D + KVD;
    if (e.rope && !is_v) {
        const float2 cs = sh.cs[col][(row % hd) >> 1];    // src/model.c:137-166
        const float n0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
        const float n1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
        v0 = n0; v1 = n1;
    }
    if (row < D) {
        float *q = g.y + (long long)col * g.y_ld;
        q[row] = v0; q[row + 1] = v1;
        return;
    }
    const int kvr = is_v ? row - D - KVD : row - D;
    const int head = kvr / hd, dim = kvr % hd;
    const int pg = sh.cur_page[col];
    if (pg < 0 || pg >= e.n_pages) {   // never write outside the pool
        if (g.fault) atomicExch(g.fault, FAULT_BAD_PAGE);
        return;
    }
    const int t = pos % e.page_tokens;
    float *base = e.kv_pages + (long long)pg * e.page_floats +
                  ((((long long)e.layer * 2 + (is_v ? 1 : 0)) * e.n_kv + head) * e.page_tokens + t) * hd + dim;
    base[0] = v0; base[1] = v1;
    fence_proxy_async_global();   // read back by the attention items' bulk copies
}

// Tile geometry: warps = (row group rg, K part kp); short tiles split K.
struct DsTile {
    int r0, nrow, rgroups, kw, rg, kp, row0;
    bool active;
};

__device__ __forceinline__ DsTile ds_tile(int rb, int re, int ti, int warp) {
    DsTile t;
    t.r0 = rb + ti * DS_TR;
    t.nrow = min(DS_TR, re - t.r0);
    t.rgroups = (t.nrow + DS_R - 1) / DS_R;
    t.kw = t.rgroups <= 1 ? 8 : t.rgroups <= 2 ? 4 : t.rgroups <= 4 ? 2 : 1;
    t.rg = warp % t.rgroups;
    t.kp = warp / t.rgroups;
    t.active = t.kp < t.kw;
    t.row0 = t.r0 + t.rg * DS_R;
    return t;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

template <int DT, int NC>
__device__ void ds_gemv(const DsArgs &a, const DsPhase *ph, uint8_t *ring, uint64_t *full, uint64_t *empty,
                        uint8_t *uni, DsShared &sh, uint32_t &seq, int tid, unsigned long long *sub) {
    constexpr int VPC = Fmt<DT>::VPC;
    constexpr int CR = Fmt<DT>::CR;
    const int lane = tid & 31, warp = tid >> 5;
    GemvArgs g = ph->g;
    g.ncol = a.ncol;
    g.fault = a.fault;
    const int epi = ph->epi;
    const int K = g.w.k;
    const int C = K / VPC;
    const int CP = gemv_chunks_padded(K, VPC);
    float4 *XS = reinterpret_cast<float4 *>(uni);
    float *RS = reinterpret_cast<float *>(XS + (size_t)NC * CP * CR * 4);
    int rb, re;
    ds_rows(g, rb, re);
    const int ntile = (re - rb + DS_TR - 1) / DS_TR;
    if (ntile == 0) return;   // no rows of this phase here (the producer skips it too)

    // residual rows of the first tile: start their loads before anything else
    float old = 0.f;
    auto resid_load = [&](const DsTile &t) {
        if (epi == EPI_RESID && t.active && t.kp == 0 && lane < DS_R * NC) {
            const int r = lane / NC, col = lane % NC, row = t.row0 + r;
            if (row < g.w.rows && col < g.ncol) old = __ldcg(g.y + (long long)col * g.y_ld + row);
        }
    };
    resid_load(ds_tile(rb, re, 0, warp));

    // ---- activations: one read of x into the interleaved layout ------------
    //   XS[col][c / 32][p][i][c % 32] (float4), RS[col][c / 32][p][c % 32]
    float ss[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) ss[c] = 0.f;
    for (int j = tid; j < NC * C * CR; j += DS_CTHREADS) {
        const int col = j / (C * CR), rem = j % (C * CR), c = rem / CR, p = rem % CR;
        int q0, q1;
        chunk_runs<DT>(c, q0, q1);
        const int r = p ? q1 : q0;
        float v[16];
        const float *src = g.x + (long long)col * g.x_ld + r;
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = col < g.ncol ? __ldcg(src + i) : 0.f;
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) t = __fmaf_rn(v[i], v[i], t);
#pragma unroll
        for (int c2 = 0; c2 < NC; c2++) if (c2 == col) ss[c2] += t;
        float4 *dst = XS + ((size_t)col * CP * CR * 4 + (size_t)(c >> 5) * CR * 32 * 4 + (size_t)p * 4 * 32) + (c & 31);
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    const float *nw = nullptr;
    uint32_t nslot_used = 0;
    if (g.norm_w) {
        // RMS of each column (src/model.c:90-97)
#pragma unroll
        for (int c = 0; c < NC; c++) {
            float v = warp_sum(ss[c]);
            if (lane == 0) sh.red_ss[warp][c] = v;
        }
        named_bar_sync(1, DS_CTHREADS);
        if (tid < NC) {
            float t = 0.f;
            for (int w = 0; w < DS_CWARPS; w++) t += sh.red_ss[w][tid];
            sh.inv_rms[tid] = 1.0f / sqrtf(t / (float)K + g.eps);
        }
        // the gains, from the ring slot the producer filled for this phase
        nslot_used = seq % (uint32_t)a.nslot;
        mbar_wait(&full[nslot_used], (seq / (uint32_t)a.nslot) & 1, a.fault, FAULT_GEMV_FULL);
        nw = reinterpret_cast<const float *>(ring + (size_t)nslot_used * a.slot_bytes);
    }
    named_bar_sync(1, DS_CTHREADS);
    // pass 2 in shared memory: normalise, scale by 2^85, run sums
    for (int j = tid; j < NC * C * CR; j += DS_CTHREADS) {
        const int col = j / (C * CR), rem = j % (C * CR), c = rem / CR, p = rem % CR;
        int q0, q1;
        chunk_runs<DT>(c, q0, q1);
        const int r = p ? q1 : q0;
        float4 *dst = XS + ((size_t)col * CP * CR * 4 + (size_t)(c >> 5) * CR * 32 * 4 + (size_t)p * 4 * 32) + (c & 31);
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 f = dst[i * 32];
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        if (nw) {
            const float ir = sh.inv_rms[col];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __fmul_rn(nw[r + i], __fmul_rn(v[i], ir));
        }
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i++) { v[i] *= kXScale; t += v[i]; }
#pragma unroll
        for (int i = 0; i < 4; i++) dst[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        RS[(size_t)col * CP * CR + (size_t)(c >> 5) * CR * 32 + p * 32 + (c & 31)] = t * __int_as_float(1);
    }
    named_bar_sync(1, DS_CTHREADS);
    if (g.norm_w) {
        if (lane == 0) mbar_arrive(&empty[nslot_used]);
        seq++;
    }
    if (sub && tid == 0) sub[0] = globaltimer_ns();

    // ---- weights from the ring ----------------------------------------------
    int kbuf = 0;
    for (int ti = 0; ti < ntile; ti++) {
        const DsTile t = ds_tile(rb, re, ti, warp);
        if (ti > 0) resid_load(t);
        float acc[DS_R * NC];
#pragma unroll
        for (int i = 0; i < DS_R * NC; i++) acc[i] = 0.f;
        for (int kci = 0; kci < g.w.nkc; kci++, seq++) {
            const uint32_t s = seq % (uint32_t)a.nslot, n = seq / (uint32_t)a.nslot;
            mbar_wait(&full[s], n & 1, a.fault, FAULT_GEMV_FULL);   // a timeout is caught at the next grid sync
            if (sub && tid == 0 && ti == 0 && kci == 0) sub[1] = globaltimer_ns();
            const uint8_t *stage = ring + (size_t)s * a.slot_bytes;
            const int CC = qw_chunk_values(g.w, kci) / VPC;
            const int c0 = kci * (g.w.kc / VPC);
            int st[4];
#pragma unroll
            for (int p = 0; p < 4; p++) st[p] = qw_stride(g.w, p, kci);
            if (t.active) {
                for (int cl = lane + 32 * t.kp; cl < CC; cl += 32 * t.kw) {
                    const int c = c0 + cl;
#pragma unroll
                    for (int col = 0; col < NC; col++) {
                        const float4 *xb = XS + (size_t)col * CP * CR * 4 + (size_t)(c >> 5) * CR * 32 * 4 + (c & 31);
                        const float *rbp = RS + (size_t)col * CP * CR + (size_t)(c >> 5) * CR * 32 + (c & 31);
                        float4 x0[4], x1[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) x0[i] = xb[i * 32];
                        const float s0 = rbp[0];
                        float s1 = s0;
                        if constexpr (CR == 2) {
#pragma unroll
                            for (int i = 0; i < 4; i++) x1[i] = xb[(4 + i) * 32];
                            s1 = rbp[32];
                        } else {
#pragma unroll
                            for (int i = 0; i < 4; i++) x1[i] = x0[i];
                        }
#pragma unroll
                        for (int r = 0; r < DS_R; r++)
                            acc[r * NC + col] += chunk_math<DT>(stage, g.pc, st, t.rg * DS_R + r, cl, c, x0, x1, s0, s1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (sub && tid == 0 && ti == ntile - 1) sub[2] = globaltimer_ns();
        float vals[DS_R * NC];
#pragma unroll
        for (int i = 0; i < DS_R * NC; i++) vals[i] = warp_sum(acc[i]);
        if (t.kw > 1) {
            if (t.active && t.kp > 0 && lane == 0) {
#pragma unroll
                for (int i = 0; i < DS_R * NC; i++) sh.kred[kbuf][warp][i] = vals[i];
            }
            named_bar_sync(1, DS_CTHREADS);
            if (t.active && t.kp == 0) {
                for (int q = 1; q < t.kw; q++) {
#pragma unroll
                    for (int i = 0; i < DS_R * NC; i++) vals[i] += sh.kred[kbuf][t.rg + q * t.rgroups][i];
                }
            }
            kbuf ^= 1;
        }
        if (t.active && t.kp == 0 && t.row0 < re) {
#pragma unroll
            for (int i = 0; i < DS_R * NC; i++) vals[i] *= final_scale<DT>();
            switch (epi) {
            case EPI_STORE:  gemv_epilogue<NC, DS_R, EPI_STORE>(g, t.row0, vals, lane); break;
            case EPI_SWIGLU: gemv_epilogue<NC, DS_R, EPI_SWIGLU>(g, t.row0, vals, lane); break;
            case EPI_RESID:
                if (lane < DS_R * NC) {   // x += sublayer out (src/model.c:232,259)
                    const int r = lane / NC, col = lane % NC, row = t.row0 + r;
                    if (row < g.w.rows && col < g.ncol) g.y[(long long)col * g.y_ld + row] = old + vals[lane];
                }
                break;
            default: ds_epi_qkv<NC>(g, sh, t.row0, vals, lane); break;
            }
        }
    }
    if (sub && tid == 0) sub[3] = globaltimer_ns();
}

// Attention items of this CTA: the active (column, kv head, split) items of
// the step, dealt round robin over the grid.
__device__ void ds_attention(const DsArgs &a, int layer, float *sm, const int *pages, uint64_t *abar,
                             uint32_t &apar, DsShared &sh, int tid) {
    AttnArgs at = a.attn;
    at.layer = layer;
    const int S = at.split_tokens;
    int cnt[DS_MAX_NC];
    int total = 0;
#pragma unroll
    for (int c = 0; c < DS_MAX_NC; c++) {
        const int pos = c < a.ncol ? sh.pos[c] : -1;
        cnt[c] = pos < 0 ? 0 : at.n_kv * (pos / S + 1);
        total += cnt[c];
    }
    for (int i = blockIdx.x; i < total; i += gridDim.x) {
        int col = 0, r = i;
        while (r >= cnt[col]) { r -= cnt[col]; col++; }
        const int nsp = cnt[col] / at.n_kv;
        const int hk = r / nsp, s = r % nsp;
        const int *pt = pages + (size_t)col * at.max_pages;
        bool ok = at.d_head == 64 ? attn_item<2>(at, s, hk, col, sh.pos[col], pt, sm, abar, apar, sh.at, tid)
                                  : attn_item<4>(at, s, hk, col, sh.pos[col], pt, sm, abar, apar, sh.at, tid);
        if (!ok) return;   // fault recorded; the next grid sync stops the step
    }
}

// Per-step constants into shared memory: positions, page-table rows (the
// part up to each position), the page of the current token and the RoPE row.
__device__ void ds_step_constants(const DsArgs &a, int *pages, DsShared &sh, int tid) {
    const AttnArgs &at = a.attn;
    __shared__ int srow[DS_MAX_NC];
    if (tid < DS_MAX_NC) {
        const int pos = tid < a.ncol ? __ldcg(at.pos + tid) : -1;
        sh.pos[tid] = pos;
        srow[tid] = (tid < a.ncol && at.slot) ? __ldcg(at.slot + tid) : tid;
    }
    named_bar_sync(1, DS_CTHREADS);
    const int half = at.d_head / 2;
    for (int i = tid; i < a.ncol * at.max_pages; i += DS_CTHREADS) {
        const int c = i / at.max_pages, k = i % at.max_pages;
        const int pos = sh.pos[c];
        pages[i] = (pos >= 0 && k <= pos / at.page_tokens)
                       ? __ldcg(at.page_table + (long long)srow[c] * at.max_pages + k) : -1;
    }
    for (int i = tid; i < a.ncol * half; i += DS_CTHREADS) {
        const int c = i / half, k = i % half;
        const int pos = sh.pos[c];
        sh.cs[c][k] = (pos >= 0 && a.rope_cs) ? __ldg(a.rope_cs + (long long)pos * half + k) : make_float2(1.f, 0.f);
    }
    named_bar_sync(1, DS_CTHREADS);
    if (tid < DS_MAX_NC) {
        const int pos = sh.pos[tid];
        sh.cur_page[tid] = (tid < a.ncol && pos >= 0) ? pages[(size_t)tid * at.max_pages + pos / at.page_tokens] : -1;
    }
    named_bar_sync(1, DS_CTHREADS);
}

template <int NC>
__global__ void __launch_bounds__(DS_THREADS, 1) k_decode(const __grid_constant__ DsArgs a) {
    uint8_t *ring = cmolcu_smem;
    uint8_t *uni = ring + (size_t)a.nslot * a.slot_bytes;
    int *pages = reinterpret_cast<int *>(uni + a.union_bytes);                    // [NC][max_pages]
    uint64_t *bars = reinterpret_cast<uint64_t *>(uni + a.union_bytes + a.pages_bytes);
    uint64_t *full = bars, *empty = bars + DS_MAX_SLOTS, *abar = bars + 2 * DS_MAX_SLOTS;
    __shared__ DsShared sh;
    const int tid = threadIdx.x, warp = tid >> 5;

    if (tid == 0) {
        for (int s = 0; s < a.nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], DS_CWARPS);
        }
        mbar_init(abar, 1);
        fence_mbar_init();
        sh.abort = 0;
    }
    __syncthreads();
    pdl_launch_dependents();
    if (warp == DS_CWARPS) {
        ds_producer(a, ring, full, empty, sh, tid & 31);
        return;
    }
    pdl_wait();   // x, the page table and the barrier counter come from the step-begin kernel
    ds_step_constants(a, pages, sh, tid);

    uint32_t seq = 0, apar = 0;
    unsigned int nsync = 0;
    const bool tr = a.trace && blockIdx.x == 0 && tid == 0;
    if (tr) a.trace[0] = globaltimer_ns();
    for (int p = 0; p < a.n_phases; p++) {
        const DsPhase *ph = a.phases + p;
        unsigned long long *sub = (a.trace && blockIdx.x == 0) ? a.trace + 2 * a.n_phases + 1 + 4 * p : nullptr;
        if (ph->kind == DS_GEMV) {
            switch (ph->g.w.dtype) {
            case DT_Q4_0: ds_gemv<DT_Q4_0, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            case DT_Q5_0: ds_gemv<DT_Q5_0, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            case DT_Q8_0: ds_gemv<DT_Q8_0, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            case DT_Q4_K: ds_gemv<DT_Q4_K, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            case DT_Q6_K: ds_gemv<DT_Q6_K, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            case DT_F16:  ds_gemv<DT_F16, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            default:      ds_gemv<DT_F32, NC>(a, ph, ring, full, empty, uni, sh, seq, tid, sub); break;
            }
        } else {
            ds_attention(a, ph->layer, reinterpret_cast<float *>(uni), pages, abar, apar, sh, tid);
        }
        if (tr) a.trace[2 * p + 1] = globaltimer_ns();
        if (p + 1 < a.n_phases) {
            nsync++;
            if (!ds_grid_sync(a.sync_count, nsync * gridDim.x, a.fault, tid, sh)) return;
        }
        if (tr) a.trace[2 * p + 2] = globaltimer_ns();
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef void (*ds_kernel_t)(DsArgs);

static ds_kernel_t ds_pick(int nc) {
    switch (nc) {
    case 1: return k_decode<1>;
    case 2: return k_decode<2>;
    case 4: return k_decode<4>;
    default: return nullptr;
    }
}

static void ds_fmt(int dt, int &vpc, int &cr) {
    vpc = (dt == DT_Q8_0 || dt == DT_F16 || dt == DT_F32) ? 16 : 32;
    cr = vpc == 16 ? 1 : 2;
}

void ds_partition(DsPhase *ph, int n, int grid) {
    for (int i = 0; i < n; i++) {
        if (ph[i].kind != DS_GEMV) continue;
        QWeight &w = ph[i].g.w;
        PipeCfg &pc = ph[i].g.pc;
        int rpc = (w.rows + grid - 1) / grid;
        pc.rows_per_cta = (rpc + DS_R - 1) / DS_R * DS_R;
        int off = 0;
        for (int p = 0; p < 4; p++) {
            pc.po[p] = off;
            off += p < w.nplanes ? DS_TR * w.cs[p] : 0;
        }
        pc.sb = off;
        pc.nstage = 0;
    }
}

static bool ds_fail(const char *why, int v) {
    const char *e = getenv("CMOLCU_VERBOSE");
    if (e && e[0] == '1') fprintf(stderr, "[cmolcu] step kernel plan: %s (%d)\n", why, v);
    return false;
}

bool ds_plan(const DsPhase *ph, int n, int nc, int d_head, int G, int split_tokens, int max_pages,
             DsPlan &plan) {
    ds_kernel_t k = ds_pick(nc);
    if (!k || (d_head != 64 && d_head != 128) || G > ATTN_MAX_G) return ds_fail("shape", d_head);
    size_t slot = 0, uni = attn_item_smem_bytes(d_head, G, split_tokens);
    for (int i = 0; i < n; i++) {
        if (ph[i].kind != DS_GEMV) continue;
        const QWeight &w = ph[i].g.w;
        if (w.k > CMOLCU_GEMV_MAX_K || w.k % 16) return ds_fail("k", w.k);
        int vpc, cr;
        ds_fmt(w.dtype, vpc, cr);
        slot = std::max(slot, (size_t)ph[i].g.pc.sb);
        if (ph[i].g.norm_w) slot = std::max(slot, (size_t)w.k * 4);
        uni = std::max(uni, gemv_x_bytes(nc, w.k, vpc, cr));
    }
    slot = (slot + 127) & ~(size_t)127;
    uni = (uni + 127) & ~(size_t)127;
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa = {};
    cudaError_t fe = cudaFuncGetAttributes(&fa, k);
    if (fe != cudaSuccess) { cudaGetLastError(); return ds_fail("cudaFuncGetAttributes", (int)fe); }
    const size_t bars = (2 * DS_MAX_SLOTS + 1) * 8;
    const size_t pages = ((size_t)nc * max_pages * 4 + 127) & ~(size_t)127;
    const long long room =
        (long long)optin - (long long)fa.sharedSizeBytes - (long long)uni - (long long)pages - (long long)bars;
    if (slot == 0 || room < 2 * (long long)slot) return ds_fail("shared memory room", (int)room);
    const int nslot = (int)std::min<long long>(DS_MAX_SLOTS, room / (long long)slot);
    plan.nc = nc;
    plan.nslot = nslot;
    plan.slot_bytes = (int)slot;
    plan.union_bytes = (int)uni;
    plan.pages_bytes = (int)pages;
    plan.smem = (size_t)nslot * slot + uni + pages + bars;
    fe = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
    if (fe != cudaSuccess) { cudaGetLastError(); return ds_fail("cudaFuncSetAttribute", (int)fe); }
    // the occupancy query (and the launch) follow the kernel's carveout: ask for all-shared
    fe = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    if (fe != cudaSuccess) { cudaGetLastError(); return ds_fail("carveout", (int)fe); }
    int per_sm = 0;
    fe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, DS_THREADS, plan.smem);
    if (fe != cudaSuccess || per_sm < 1) { cudaGetLastError(); return ds_fail("occupancy", fe != cudaSuccess ? (int)fe : per_sm); }
    plan.grid = device_sm_count();
    return true;
}

cudaError_t ds_launch(const DsArgs &a0, const DsPlan &plan, int d_head, cudaStream_t st, bool pdl) {
    (void)d_head;
    ds_kernel_t k = ds_pick(plan.nc);
    if (!k || a0.ncol < 1 || a0.ncol > plan.nc) return cudaErrorInvalidValue;
    DsArgs a = a0;
    a.nslot = plan.nslot;
    a.slot_bytes = plan.slot_bytes;
    a.union_bytes = plan.union_bytes;
    a.pages_bytes = plan.pages_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeCooperative;       // every CTA resident: the grid barrier needs it
    attr[na].val.cooperative = 1;
    na++;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, a);
}
