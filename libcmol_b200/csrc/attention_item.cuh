// attention_item.cuh — one work item of split-context GQA decode attention
// (the kernels of attention.cu run it).
//
// Item = (context split s, kv head hk, column col), run by ATTN_THREADS
// threads that synchronise on named barrier 1.  Thread 0 moves the K and V
// blocks of the split's pages (each a contiguous page_tokens x d_head block
// in the page layout) into shared memory with cp.async.bulk on one mbarrier
// while the others load the G = n_heads / n_kv queries.  Scores: one thread
// per (token, head).  Softmax per head.  P.V: (head, float4 of d_head) items
// with the split's tokens divided among thread groups.  The partial (max,
// sum, acc) goes to a.part; the last item of a (column, kv head) to finish —
// found with an atomic counter — merges the partials in split order (so the
// result does not depend on scheduling) and resets the counter.
// Replaces step 5 of cmol_attn_forward (src/attn.c:103-137).
#pragma once
#include "attention.cuh"
#include "sync.cuh"

#define ATTN_WARPS 8
#define ATTN_THREADS (ATTN_WARPS * 32)
#define ATTN_MAX_G 8

struct AttnShared {
    float wsum[ATTN_MAX_G], wmax[ATTN_MAX_G];
    int   last, ok;
};

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Shared-memory bytes of one item (K and V tiles of kvb-byte values,
// queries, scores, P.V sums).
__host__ __device__ inline size_t attn_item_smem_bytes(int d_head, int G, int split_tokens, int kvb) {
    return (size_t)2 * split_tokens * d_head * kvb + (size_t)G * d_head * 4 + (size_t)G * split_tokens * 4 +
           (size_t)ATTN_THREADS * 16;
}

// Values 4c .. 4c+3 of row t (context position pos) of a shared-memory K or
// V tile of hd-value rows, as floats: f32 tiles directly, f16 tiles (whose
// 16-byte chunks are swizzled by position, kv_swz) widened exactly.
template <bool H, int HD>
__device__ __forceinline__ float4 kv4(const unsigned char *tile, int t, int pos, int c) {
    if constexpr (H) {
        const uint2 u = *reinterpret_cast<const uint2 *>(tile + ((size_t)t * HD + kv_swz(pos, 4 * c, HD)) * 2);
        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
        return reinterpret_cast<const float4 *>(tile)[(size_t)t * (HD / 4) + c];
    }
}

// `sm` is 16-byte aligned; `bar` an initialised mbarrier (count 1) whose
// next phase has parity `parity` (toggled here when the item waits on it).
// Returns false when a wait ran out (fault word set); every thread returns
// the same value at the same point.
// `pos` is the column's position (< 0: inactive) and `pt` its page-table row
// (global or shared memory).  H: the KV pool holds f16 values.
template <int E, bool H>
__device__ bool attn_item(const AttnArgs &a, int s, int hk, int col, int pos, const int *pt, float *sm,
                          uint64_t *bar, uint32_t &parity, AttnShared &sh, int tid) {
    constexpr int hd = 32 * E, HD4 = hd / 4;
    constexpr int KB = H ? 2 : 4;                // bytes per K / V value
    const int lane = tid & 31, warp = tid >> 5;
    const int G = a.n_heads / a.n_kv;
    const int S = a.split_tokens;
    const int P = a.page_tokens;

    unsigned char *Ks = reinterpret_cast<unsigned char *>(sm);                 // [S][hd] values
    unsigned char *Vs = Ks + (size_t)S * hd * KB;                                // [S][hd] values
    float *Qs = reinterpret_cast<float *>(Vs + (size_t)S * hd * KB);             // [G][hd]
    float *Sc = Qs + (size_t)G * hd;                                            // [G][S]
    float4 *Red = reinterpret_cast<float4 *>(Sc + (size_t)G * S);               // [ATTN_THREADS]
    const unsigned char *pool = static_cast<const unsigned char *>(a.kv_pages);

    if (pos < 0) return true;
    const int t0 = s * S;
    if (t0 > pos) return true;
    const int n = min(S, pos + 1 - t0);                       // tokens in this split
    const int n_active = (pos + S) / S;
    const long long head_off = (long long)hk * 2 * P * hd;   // the kv head's K block in the layer's page
    const long long v_off = (long long)P * hd;                            // V block follows

    if (tid == 0) {
        int ok = 1;
        const int npg = (n + P - 1) / P;
        for (int i = 0; i < npg; i++) {
            int pg = pt[t0 / P + i];
            if (pg < 0 || pg >= a.n_pages) ok = 0;
        }
        if (ok) {
            // the KV rows of this step were written through the generic proxy
            fence_proxy_async_global();
            mbar_arrive_expect_tx(bar, (uint32_t)(2 * npg * P * hd * KB));
            for (int i = 0; i < npg; i++) {
                const unsigned char *kp = pool + ((long long)pt[t0 / P + i] * a.page_elems + head_off) * KB;
                bulk_g2s(Ks + (size_t)i * P * hd * KB, kp, (uint32_t)(P * hd * KB), bar);
                bulk_g2s(Vs + (size_t)i * P * hd * KB, kp + v_off * KB, (uint32_t)(P * hd * KB), bar);
            }
        } else if (a.fault) {
            atomicExch(a.fault, FAULT_BAD_PAGE);
        }
        sh.ok = ok;
    }
    __syncwarp();   // warp 0 re-converges before the CTA barrier (which counts whole warps)
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
        Qs[i] = __ldcg(a.q + (long long)col * a.q_ld + (long long)hk * G * hd + i);
    named_bar_sync(1, ATTN_THREADS);
    if (!sh.ok) return false;
    const bool got = mbar_wait(bar, parity, a.fault, FAULT_ATTN_WAIT);
    parity ^= 1u;
    if (!got) sh.ok = 0;
    named_bar_sync(1, ATTN_THREADS);
    if (!sh.ok) return false;

    // scores: one thread per (token, head).  Lane l starts its walk over the
    // row at float4 l % HD4, so the 8 lanes of a shared-memory phase touch 8
    // different 16-byte bank groups of their (different) K rows.
    {
        const float4 *Q4 = reinterpret_cast<const float4 *>(Qs);
        for (int w = tid; w < n * G; w += ATTN_THREADS) {
            const int t = w % n, g = w / n;
            const float4 *qr = Q4 + (size_t)g * HD4;
            float d0 = 0.f, d1 = 0.f;
#pragma unroll
            for (int j = 0; j < HD4; j++) {
                const int c = (j + lane) & (HD4 - 1);
                const float4 k = kv4<H, hd>(Ks, t, t0 + t, c), q = qr[c];
                d0 = __fmaf_rn(q.x, k.x, d0);
                d1 = __fmaf_rn(q.y, k.y, d1);
                d0 = __fmaf_rn(q.z, k.z, d0);
                d1 = __fmaf_rn(q.w, k.w, d1);
            }
            Sc[g * S + t] = (d0 + d1) * a.scale;
        }
    }
    named_bar_sync(1, ATTN_THREADS);
    // per-head softmax over the split (max, exp, sum)
    for (int g = warp; g < G; g += ATTN_WARPS) {
        float m = -INFINITY;
        for (int t = lane; t < n; t += 32) m = fmaxf(m, Sc[g * S + t]);
        m = warp_max(m);
        float sum = 0.f;
        for (int t = lane; t < n; t += 32) {
            float e = expf(Sc[g * S + t] - m);
            Sc[g * S + t] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) { sh.wmax[g] = m; sh.wsum[g] = sum; }
    }
    named_bar_sync(1, ATTN_THREADS);
    // P.V: item = (head, float4 of d_head); the split's tokens are divided
    // among `parts` thread groups whose float4 sums meet in shared memory.
    {
        const int items = G * HD4;   // up to 2 * ATTN_THREADS (G = 8, d_head = 256)
        const int parts = max(1, min(ATTN_THREADS / items, n));
        const int item = tid % items, part = tid / items;
        if (items > ATTN_THREADS) {
            // one thread per item over all tokens, two items per thread
            for (int it = tid; it < items; it += ATTN_THREADS) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                const int g = it / HD4, c = it % HD4;
                const float *p = Sc + g * S;
                for (int t = 0; t < n; t++) {
                    const float pt_ = p[t];
                    const float4 v = kv4<H, hd>(Vs, t, t0 + t, c);
                    acc.x = __fmaf_rn(pt_, v.x, acc.x);
                    acc.y = __fmaf_rn(pt_, v.y, acc.y);
                    acc.z = __fmaf_rn(pt_, v.z, acc.z);
                    acc.w = __fmaf_rn(pt_, v.w, acc.w);
                }
                float *pp = a.part + (((long long)col * a.n_heads + hk * G + g) * a.n_splits + s) * (hd + 2);
                pp[4 * c + 0] = acc.x;
                pp[4 * c + 1] = acc.y;
                pp[4 * c + 2] = acc.z;
                pp[4 * c + 3] = acc.w;
                if (c == 0) { pp[hd] = sh.wmax[g]; pp[hd + 1] = sh.wsum[g]; }
            }
        } else if (part < parts) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            const int g = item / HD4, c = item % HD4;
            const float *p = Sc + g * S;
            const int tb = (int)((long long)n * part / parts), te = (int)((long long)n * (part + 1) / parts);
            for (int t = tb; t < te; t++) {
                const float pt_ = p[t];
                const float4 v = kv4<H, hd>(Vs, t, t0 + t, c);
                acc.x = __fmaf_rn(pt_, v.x, acc.x);
                acc.y = __fmaf_rn(pt_, v.y, acc.y);
                acc.z = __fmaf_rn(pt_, v.z, acc.z);
                acc.w = __fmaf_rn(pt_, v.w, acc.w);
            }
            Red[tid] = acc;
        }
        named_bar_sync(1, ATTN_THREADS);
        for (int i = tid; i < items && items <= ATTN_THREADS; i += ATTN_THREADS) {
            float4 r = Red[i];
            for (int q = 1; q < parts; q++) {
                const float4 o = Red[q * items + i];
                r.x += o.x; r.y += o.y; r.z += o.z; r.w += o.w;
            }
            const int g = i / HD4, c = i % HD4;
            float *pp = a.part + (((long long)col * a.n_heads + hk * G + g) * a.n_splits + s) * (hd + 2);
            pp[4 * c + 0] = r.x;
            pp[4 * c + 1] = r.y;
            pp[4 * c + 2] = r.z;
            pp[4 * c + 3] = r.w;
            if (c == 0) { pp[hd] = sh.wmax[g]; pp[hd + 1] = sh.wsum[g]; }
        }
    }
    __threadfence();
    named_bar_sync(1, ATTN_THREADS);
    if (tid == 0) {
        int old = atomicAdd(&a.counters[col * a.n_kv + hk], 1);
        sh.last = (old == n_active - 1);
    }
    named_bar_sync(1, ATTN_THREADS);
    if (!sh.last) return true;
    __threadfence();

    // last item of (column, kv head): merge the splits in order
    for (int i = tid; i < G * hd; i += ATTN_THREADS) {
        const int g = i / hd, d = i % hd;
        const float *base = a.part + ((long long)col * a.n_heads + hk * G + g) * a.n_splits * (hd + 2);
        float M = -INFINITY;
        for (int sp = 0; sp < n_active; sp++) M = fmaxf(M, __ldcg(base + sp * (hd + 2) + hd));
        float L = 0.f, A = 0.f;
        for (int sp = 0; sp < n_active; sp++) {
            const float *pp = base + sp * (hd + 2);
            const float f = expf(__ldcg(pp + hd) - M);
            L = __fmaf_rn(__ldcg(pp + hd + 1), f, L);
            A = __fmaf_rn(__ldcg(pp + d), f, A);
        }
        a.out[(long long)col * a.out_ld + (long long)(hk * G + g) * hd + d] = A / L;
    }
    if (tid == 0) a.counters[col * a.n_kv + hk] = 0;
    // the Red / Sc buffers are reused by the next item
    named_bar_sync(1, ATTN_THREADS);
    return true;
}

// ---------------------------------------------------------------------------
// Group-aware item.  The columns of one session in a step (same page-table
// row, contiguous, consecutive positions: a prefill chunk) form a group.  The
// group's columns at positions p with (p + 1) % a.q_block == 0, and its last
// column, are leaders: the CTA of a leader serves the up to a.q_block
// queries of the group ending at it from one
// load of the split's keys and values; the other columns' CTAs return at
// once.  Each query attends causally to the split's tokens up to its own
// position.  Queries go through in chunks of `a.q_chunk` (Q and score tiles
// in shared memory).  Every query with tokens in the split writes its
// partial, and the item that completes a query's split count merges it, in
// split order.
// ---------------------------------------------------------------------------
#define ATTN_QB 32   // most queries of one leader (a warp's lanes scan them)

// Query-chunk size for a budget of `budget` bytes of query and score tiles.
__host__ __device__ inline int attn_group_qc(int d_head, int G, int split_tokens, int budget) {
    const int per_q = G * (d_head + split_tokens) * 4;
    const int qc = budget / per_q;
    return qc < 1 ? 1 : qc > ATTN_QB ? ATTN_QB : qc;
}

// K and V tiles, query and score tiles, P.V sums, per-row max / sum and
// per-query merge flags (floats, 16-byte multiple).
__host__ __device__ inline size_t attn_group_smem_bytes(int d_head, int G, int split_tokens, int qc, int kvb) {
    const size_t tail = ((size_t)2 * qc * G * 4 + (size_t)qc * 4 + 15) & ~(size_t)15;
    return (size_t)2 * split_tokens * d_head * kvb + (size_t)qc * G * d_head * 4 +
           (size_t)qc * G * split_tokens * 4 + (size_t)ATTN_THREADS * 16 + tail;
}

struct AttnGroupShared {
    int q_lo, ok;
};

// Column c (position pos_c >= 0, page-table row slot_c) belongs to a group
// of more than one column; `next` says whether column c + 1 continues it.
// a.slot is non-null.
template <int E, bool H>
__device__ bool attn_group_item(const AttnArgs &a, int s, int hk, int c, int pos_c, int slot_c, bool next, float *sm,
                                uint64_t *bar, uint32_t &parity, AttnGroupShared &gs, int tid) {
    constexpr int hd = 32 * E, HD4 = hd / 4;
    constexpr int KB = H ? 2 : 4;                // bytes per K / V value
    const int lane = tid & 31, warp = tid >> 5;
    const int G = a.n_heads / a.n_kv;
    const int S = a.split_tokens;
    const int P = a.page_tokens;
    const int QC = a.q_chunk;
    const int QB = a.q_block;

    // a column whose successor continues its group leads only at a block end
    if (next && (pos_c + 1) % QB != 0) return true;
    const int t0 = s * S;
    if (t0 > pos_c) return true;
    const int n = min(S, pos_c + 1 - t0);                     // tokens of this split the block sees

    unsigned char *Ks = reinterpret_cast<unsigned char *>(sm);  // [S][hd] values
    unsigned char *Vs = Ks + (size_t)S * hd * KB;               // [S][hd] values
    float *Qs = reinterpret_cast<float *>(Vs + (size_t)S * hd * KB);   // [QC][G][hd]
    const unsigned char *pool = static_cast<const unsigned char *>(a.kv_pages);
    float *Sc = Qs + (size_t)QC * G * hd;                     // [QC][G][S]
    float4 *Red = reinterpret_cast<float4 *>(Sc + (size_t)QC * G * S);   // [ATTN_THREADS]
    float *Wmax = reinterpret_cast<float *>(Red + ATTN_THREADS);         // [QC][G]
    float *Wsum = Wmax + QC * G;                                          // [QC][G]
    int *Merge = reinterpret_cast<int *>(Wsum + QC * G);                  // [QC]
    const int *pt = a.page_table + (long long)slot_c * a.max_pages;
    const long long head_off = (long long)hk * 2 * P * hd;
    const long long v_off = (long long)P * hd;

    if (tid == 0) {
        int ok = 1;
        const int npg = (n + P - 1) / P;
        for (int i = 0; i < npg; i++) {
            int pg = pt[t0 / P + i];
            if (pg < 0 || pg >= a.n_pages) ok = 0;
        }
        if (ok) {
            fence_proxy_async_global();   // the KV rows of this step were written through the generic proxy
            mbar_arrive_expect_tx(bar, (uint32_t)(2 * npg * P * hd * KB));
            for (int i = 0; i < npg; i++) {
                const unsigned char *kp = pool + ((long long)pt[t0 / P + i] * a.page_elems + head_off) * KB;
                bulk_g2s(Ks + (size_t)i * P * hd * KB, kp, (uint32_t)(P * hd * KB), bar);
                bulk_g2s(Vs + (size_t)i * P * hd * KB, kp + v_off * KB, (uint32_t)(P * hd * KB), bar);
            }
        } else if (a.fault) {
            atomicExch(a.fault, FAULT_BAD_PAGE);
        }
        gs.ok = ok;
    }
    if (warp == 0) {
        // the block's first query: lane k (1 <= k <= pos_c % ATTN_QB) checks
        // that column c - k continues the group; the block starts after the
        // nearest break
        const int back = pos_c % QB;
        const int q = c - lane;
        const bool brk = lane >= 1 && lane <= back && (q < 0 || a.slot[q] != slot_c || a.pos[q] != pos_c - lane);
        const unsigned m = __ballot_sync(0xffffffffu, brk);
        if (lane == 0) gs.q_lo = m ? c - (__ffs(m) - 1) + 1 : c - back;
    }
    named_bar_sync(1, ATTN_THREADS);
    if (!gs.ok) return false;
    // queries before c - (pos_c - t0) do not reach this split
    const int q_first = max(gs.q_lo, c - (pos_c - t0));
    auto load_q = [&](int qb) {
        const int rows = min(QC, c + 1 - qb) * G;
        for (int i = tid; i < rows * hd; i += ATTN_THREADS) {
            const int qi = i / (G * hd), rem = i % (G * hd);
            Qs[i] = __ldcg(a.q + (long long)(qb + qi) * a.q_ld + (long long)hk * G * hd + rem);
        }
    };
    load_q(q_first);                        // in flight with the K / V copies
    const bool got = mbar_wait(bar, parity, a.fault, FAULT_ATTN_WAIT);
    parity ^= 1u;
    if (!got) gs.ok = 0;
    named_bar_sync(1, ATTN_THREADS);
    if (!gs.ok) return false;

    for (int qb = q_first; qb <= c; qb += QC) {
        const int qn = min(QC, c + 1 - qb);
        const int rows = qn * G;
        if (qb != q_first) {
            load_q(qb);
            named_bar_sync(1, ATTN_THREADS);
        }
        // scores: one thread per (query, head, token); tokens past a query's
        // position are masked.  Lane l starts its walk over the row at float4
        // l % HD4 (distinct bank groups across the lanes of a phase).
        {
            const float4 *Q4 = reinterpret_cast<const float4 *>(Qs);
            for (int w = tid; w < rows * n; w += ATTN_THREADS) {
                const int t = w % n, row = w / n, qi = row / G;
                const int nq = min(n, pos_c - (c - (qb + qi)) + 1 - t0);   // consecutive positions
                float sc = -INFINITY;
                if (t < nq) {
                    const float4 *qr = Q4 + (size_t)row * HD4;
                    float d0 = 0.f, d1 = 0.f;
#pragma unroll
                    for (int j = 0; j < HD4; j++) {
                        const int cc = (j + lane) & (HD4 - 1);
                        const float4 k = kv4<H, hd>(Ks, t, t0 + t, cc), q = qr[cc];
                        d0 = __fmaf_rn(q.x, k.x, d0);
                        d1 = __fmaf_rn(q.y, k.y, d1);
                        d0 = __fmaf_rn(q.z, k.z, d0);
                        d1 = __fmaf_rn(q.w, k.w, d1);
                    }
                    sc = (d0 + d1) * a.scale;
                }
                Sc[row * S + t] = sc;
            }
        }
        named_bar_sync(1, ATTN_THREADS);
        // softmax of each (query, head) row over its visible tokens
        for (int row = warp; row < rows; row += ATTN_WARPS) {
            float m = -INFINITY;
            for (int t = lane; t < n; t += 32) m = fmaxf(m, Sc[row * S + t]);
            m = warp_max(m);
            float sum = 0.f;
            for (int t = lane; t < n; t += 32) {
                const float v = Sc[row * S + t];
                const float e = v == -INFINITY ? 0.f : expf(v - m);
                Sc[row * S + t] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) { Wmax[row] = m; Wsum[row] = sum; }
        }
        named_bar_sync(1, ATTN_THREADS);
        // P.V: item = (row, float4 of d_head).  Few items: the tokens are
        // divided among `parts` thread groups whose sums meet in shared memory;
        // many: one thread per item over all tokens.
        {
            const int items = rows * HD4;
            const int parts = items * 2 <= ATTN_THREADS ? max(1, min(ATTN_THREADS / items, n)) : 1;
            auto write = [&](int it, float4 r) {
                const int row = it / HD4, cc = it % HD4, qi = row / G, g = row % G;
                float *pp = a.part + (((long long)(qb + qi) * a.n_heads + hk * G + g) * a.n_splits + s) * (hd + 2);
                pp[4 * cc + 0] = r.x; pp[4 * cc + 1] = r.y; pp[4 * cc + 2] = r.z; pp[4 * cc + 3] = r.w;
                if (cc == 0) { pp[hd] = Wmax[row]; pp[hd + 1] = Wsum[row]; }
            };
            auto pv = [&](int it, int tb, int te) {
                const int row = it / HD4, cc = it % HD4;
                const float *p = Sc + row * S;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int t = tb; t < te; t++) {
                    const float pt_ = p[t];
                    const float4 v = kv4<H, hd>(Vs, t, t0 + t, cc);
                    acc.x = __fmaf_rn(pt_, v.x, acc.x);
                    acc.y = __fmaf_rn(pt_, v.y, acc.y);
                    acc.z = __fmaf_rn(pt_, v.z, acc.z);
                    acc.w = __fmaf_rn(pt_, v.w, acc.w);
                }
                return acc;
            };
            if (parts > 1) {
                const int item = tid % items, part = tid / items;
                if (part < parts)
                    Red[tid] = pv(item, (int)((long long)n * part / parts), (int)((long long)n * (part + 1) / parts));
                named_bar_sync(1, ATTN_THREADS);
                for (int i = tid; i < items; i += ATTN_THREADS) {
                    float4 r = Red[i];
                    for (int q = 1; q < parts; q++) {
                        const float4 o = Red[q * items + i];
                        r.x += o.x; r.y += o.y; r.z += o.z; r.w += o.w;
                    }
                    write(i, r);
                }
            } else {
                for (int it = tid; it < items; it += ATTN_THREADS) write(it, pv(it, 0, n));
            }
        }
        __threadfence();
        named_bar_sync(1, ATTN_THREADS);
        // count this split for each query of the chunk; merge the ones it completes
        if (tid < qn) {
            const int q = qb + tid;
            const int n_active = (pos_c - (c - q) + S) / S;
            const int old = atomicAdd(&a.counters[q * a.n_kv + hk], 1);
            Merge[tid] = (old == n_active - 1);
        }
        named_bar_sync(1, ATTN_THREADS);
        __threadfence();
        for (int qi = 0; qi < qn; qi++) {
            if (!Merge[qi]) continue;      // uniform: shared flag
            const int q = qb + qi;
            const int n_active = (pos_c - (c - q) + S) / S;
            for (int i = tid; i < G * hd; i += ATTN_THREADS) {
                const int g = i / hd, d = i % hd;
                const float *base = a.part + ((long long)q * a.n_heads + hk * G + g) * a.n_splits * (hd + 2);
                float M = -INFINITY;
                for (int sp = 0; sp < n_active; sp++) M = fmaxf(M, __ldcg(base + sp * (hd + 2) + hd));
                float L = 0.f, A = 0.f;
                for (int sp = 0; sp < n_active; sp++) {
                    const float *pp = base + sp * (hd + 2);
                    const float f = expf(__ldcg(pp + hd) - M);
                    L = __fmaf_rn(__ldcg(pp + hd + 1), f, L);
                    A = __fmaf_rn(__ldcg(pp + d), f, A);
                }
                a.out[(long long)q * a.out_ld + (long long)(hk * G + g) * hd + d] = A / L;
            }
            if (tid == 0) a.counters[q * a.n_kv + hk] = 0;
        }
        named_bar_sync(1, ATTN_THREADS);     // the tiles are reused by the next chunk
    }
    return true;
}
