// attention_decode.cuh — GQA decode attention streamed through a shared-memory
// ring: the kernel of steps whose columns are one token each (decode).
//
// Work item = CTA (chunk c of `chunk_tokens` context tokens, kv head hk,
// column col).  The chunk is cut into sub-tiles of DEC_SUB (64) tokens whose
// K and V blocks thread 0 moves into a ring of `stages` shared-memory stages
// with cp.async.bulk (one copy per page block, completion counted on the
// stage's mbarrier), so that the copies of the next sub-tiles are in flight
// while the current one is computed.  Per sub-tile:
//   scores  — warp w takes tokens w, w+8, ..., w+56; lane l holds the G
//             queries' values [E*l, E*l+E) in registers and multiplies them
//             with the same slice of each K row (one coalesced read of the
//             row per warp); the warp's 8 x G partial dot products are then
//             summed across the lanes by a reduce-scatter (each lane ends
//             with whole sums), so every K value is read from shared memory
//             once;
//   softmax — online over the chunk: per head the running max m and sum l,
//             the sub-tile's probabilities exp(s - m) and the factor
//             exp(m_old - m) that rescales the accumulators;
//   P.V     — warp w adds p(t) * V row t for its tokens into per-lane
//             accumulators (lane l: values [E*l, E*l+E) of every head).
// At the end of the chunk the 8 warps' accumulators meet in shared memory
// and the chunk's partial (acc, m, l) per head goes to a.part.  The last CTA
// of a (column, kv head) to finish — an atomic counter — merges the partials
// in chunk order (the result does not depend on scheduling) and resets the
// counter, as the split items of attention_item.cuh do.
// Replaces step 5 of cmol_attn_forward (src/attn.c:103-137): out_h =
// sum_t softmax_t(q_h . k_t / sqrt(d_head)) v_t, kv head h * n_kv / n_heads.
#pragma once
#include "attention_item.cuh"

#define DEC_SUB 64        // tokens per sub-tile
#define DEC_TPW 8         // tokens per warp per sub-tile (8 warps)
#define DEC_SHARED_BYTES 128   // DecShared, rounded up (the mbarriers follow it)

// Smallest power of two >= g (g <= 8).
__host__ __device__ constexpr int dec_pow2(int g) { return g <= 1 ? 1 : g <= 2 ? 2 : g <= 4 ? 4 : 8; }

// Shared-memory bytes of the ring and its companions (see k_attn_dec).
__host__ __device__ inline size_t dec_ring_bytes(int hd, int kvb, int stages) {
    return (size_t)stages * 2 * DEC_SUB * hd * kvb;
}
__host__ __device__ inline size_t dec_smem_bytes(int hd, int kvb, int gp, int stages) {
    size_t ring = dec_ring_bytes(hd, kvb, stages);
    const size_t red = (size_t)ATTN_WARPS * gp * hd * 4;     // end-of-chunk warp sums (alias the ring)
    if (red > ring) ring = red;
    return ring + (size_t)2 * gp * DEC_SUB * 4                 // scores [gp][SUB], probabilities [SUB][gp]
           + DEC_SHARED_BYTES + (size_t)stages * 8;             // m, l, alpha, flag; mbarriers
}

// E consecutive K or V values of a shared-memory row as floats.
template <int E, bool H>
__device__ __forceinline__ void dec_load(const unsigned char *p, float (&f)[E]) {
    if constexpr (H) {
        if constexpr (E == 4) {
            const uint2 u = *reinterpret_cast<const uint2 *>(p);
            const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
            f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
        } else {
            const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(p));
            f[0] = a.x; f[1] = a.y;
        }
    } else {
        if constexpr (E == 4) {
            const float4 u = *reinterpret_cast<const float4 *>(p);
            f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
        } else {
            const float2 u = *reinterpret_cast<const float2 *>(p);
            f[0] = u.x; f[1] = u.y;
        }
    }
}

// Reduce-scatter of C values per lane over the lanes whose bit O (and the
// lower bits) still differ: at each level a lane keeps the half of its
// values selected by its lane bit and adds the partner's copy of that half.
// With C <= 32 values the levels left after C reaches 1 sum plainly, so the
// lanes end with the total of value index lane >> (5 - log2 C); with C = 64
// each lane ends with indices 2*lane and 2*lane + 1 in v[0], v[1].
template <int C, int O>
struct DecRS {
    static __device__ __forceinline__ void run(float *v, int lane) {
        if constexpr (O == 0) {
            return;
        } else if constexpr (C == 1) {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], O);
            DecRS<1, O / 2>::run(v, lane);
        } else {
            const bool up = (lane & O) != 0;
#pragma unroll
            for (int i = 0; i < C / 2; i++) {
                const float send = up ? v[i] : v[i + C / 2];
                const float keep = up ? v[i + C / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
            }
            DecRS<C / 2, O / 2>::run(v, lane);
        }
    }
};

struct DecShared {
    float m[8], l[8], alpha[8];
    int   fail;
};

// Issues the bulk copies of sub-tile j of the chunk into its stage (thread 0).
// Returns false (copies not issued, fault word set) when a page index is
// outside the pool.
template <int E, bool H>
__device__ __forceinline__ bool dec_issue(const AttnArgs &a, const int *pt, int c0, int ntok, int j,
                                          unsigned char *stage, uint64_t *bar) {
    constexpr int hd = 32 * E, KB = H ? 2 : 4;
    const int P = a.page_tokens;
    const int t0 = c0 + j * DEC_SUB;
    const int n = min(DEC_SUB, c0 + ntok - t0);
    const int npg = (n + P - 1) / P;
    for (int i = 0; i < npg; i++) {
        const int pg = pt[t0 / P + i];
        if (pg < 0 || pg >= a.n_pages) {
            if (a.fault) atomicExch(a.fault, FAULT_BAD_PAGE);
            return false;
        }
    }
    const long long head_off = ((long long)a.layer * 2 * a.n_kv + blockIdx.y) * P * hd;
    const long long v_off = (long long)a.n_kv * P * hd;
    const unsigned char *pool = static_cast<const unsigned char *>(a.kv_pages);
    const uint32_t blk = (uint32_t)(P * hd * KB);
    mbar_arrive_expect_tx(bar, 2u * npg * blk);
    for (int i = 0; i < npg; i++) {
        const unsigned char *kp = pool + ((long long)pt[t0 / P + i] * a.page_elems + head_off) * KB;
        bulk_g2s(stage + (size_t)i * blk, kp, blk, bar);
        bulk_g2s(stage + (size_t)DEC_SUB * hd * KB + (size_t)i * blk, kp + v_off * KB, blk, bar);
    }
    return true;
}

// Grid (chunk, kv head, column), ATTN_THREADS threads.  GP = dec_pow2(G).
template <int E, bool H, int GP>
__global__ void __launch_bounds__(ATTN_THREADS, 2) k_attn_dec(AttnArgs a, int stages) {
    constexpr int hd = 32 * E, KB = H ? 2 : 4;
    constexpr int NV = DEC_TPW * GP;                    // partial dot products per lane
    constexpr int NR = NV > 32 ? NV / 32 : 1;           // whole sums per lane after the reduce-scatter
    constexpr int LV = NV <= 8 ? 3 : NV <= 16 ? 4 : NV <= 32 ? 5 : 6;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.n_heads / a.n_kv;
    const int chunk = blockIdx.x, hk = blockIdx.y, col = blockIdx.z;
    const size_t stage_bytes = (size_t)2 * DEC_SUB * hd * KB;

    unsigned char *ring = cmolcu_smem;
    size_t ring_sz = dec_ring_bytes(hd, KB, stages);
    if ((size_t)ATTN_WARPS * GP * hd * 4 > ring_sz) ring_sz = (size_t)ATTN_WARPS * GP * hd * 4;
    float *Sc = reinterpret_cast<float *>(ring + ring_sz);             // [GP][SUB]
    float *Pt = Sc + GP * DEC_SUB;                                     // [SUB][GP]
    DecShared &sh = *reinterpret_cast<DecShared *>(Pt + DEC_SUB * GP);
    static_assert(sizeof(DecShared) <= DEC_SHARED_BYTES, "DecShared outgrew its slot");
    uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(&sh) + DEC_SHARED_BYTES);

    pdl_wait();
    const int pos = a.pos[col];
    const int CH = a.chunk_tokens;
    if (pos < 0 || chunk * CH > pos) return;            // uniform over the CTA
    const int c0 = chunk * CH;
    const int ntok = min(CH, pos + 1 - c0);
    const int nsub = (ntok + DEC_SUB - 1) / DEC_SUB;
    const int n_active = (pos + CH) / CH;
    const int srow = a.slot ? a.slot[col] : col;
    const int *pt = a.page_table + (long long)srow * a.max_pages;

    int issued = 0;                                     // thread 0 only
    if (tid == 0) {
        for (int s = 0; s < stages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
        sh.fail = 0;
        // the KV rows of this step were written through the generic proxy
        fence_proxy_async_global();
        for (; issued < nsub && issued < stages; issued++)
            if (!dec_issue<E, H>(a, pt, c0, ntok, issued, ring + (size_t)issued * stage_bytes, &bars[issued])) {
                sh.fail = 1;
                break;
            }
    }
    if (tid < GP) { sh.m[tid] = -INFINITY; sh.l[tid] = 0.f; sh.alpha[tid] = 0.f; }
    // padded heads (G < GP) keep probability 0
    for (int i = tid; i < DEC_SUB * GP; i += ATTN_THREADS) Pt[i] = 0.f;

    // this lane's slice of the G queries
    float q[GP][E];
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < E; e++)
            q[g][e] = g < G ? __ldcg(a.q + (long long)col * a.q_ld + (long long)(hk * G + g) * hd + E * lane + e)
                            : 0.f;
    float acc[GP][E];
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < E; e++) acc[g][e] = 0.f;
    __syncthreads();

    int j = 0;
    for (; j < nsub; j++) {
        const int st = j % stages;
        const unsigned char *Ks = ring + (size_t)st * stage_bytes;
        const unsigned char *Vs = Ks + (size_t)DEC_SUB * hd * KB;
        const int n = min(DEC_SUB, ntok - j * DEC_SUB);
        // A failed issue (thread 0, end of an earlier iteration) is seen here
        // by some threads only, so it just saves them the wait; every thread
        // leaves the loop together at the check after the next barrier.
        if (!sh.fail && !mbar_wait(&bars[st], (uint32_t)((j / stages) & 1), a.fault, FAULT_ATTN_WAIT)) sh.fail = 1;

        // ---- scores -------------------------------------------------------
        float v[NV];
#pragma unroll
        for (int k = 0; k < DEC_TPW; k++) {
            float kf[E];
            dec_load<E, H>(Ks + ((size_t)(warp + 8 * k) * hd + E * lane) * KB, kf);
#pragma unroll
            for (int g = 0; g < GP; g++) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) d = __fmaf_rn(q[g][e], kf[e], d);
                v[k * GP + g] = d;
            }
        }
        DecRS<NV, 16>::run(v, lane);
#pragma unroll
        for (int r = 0; r < NR; r++) {
            int idx;
            bool writer;
            if constexpr (LV <= 5) {
                idx = lane >> (5 - LV);
                writer = (lane & ((1 << (5 - LV)) - 1)) == 0;
            } else {
                idx = lane * NR + r;
                writer = true;
            }
            if (writer) {
                const int k = idx / GP, g = idx % GP, t = warp + 8 * k;
                Sc[g * DEC_SUB + t] = t < n ? v[r] * a.scale : -INFINITY;
            }
        }
        named_bar_sync(1, ATTN_THREADS);
        if (sh.fail) break;                             // uniform: set before the barrier

        // ---- online softmax, one warp per head ------------------------------
        if (warp < G) {
            const int g = warp;
            const float s0 = Sc[g * DEC_SUB + lane], s1 = Sc[g * DEC_SUB + lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float m_old = sh.m[g];
            const float m_new = fmaxf(m_old, mx);
            const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
            const float sum = warp_sum(p0 + p1);
            Pt[lane * GP + g] = p0;
            Pt[(lane + 32) * GP + g] = p1;
            if (lane == 0) {
                const float al = expf(m_old - m_new);
                sh.alpha[g] = al;
                sh.m[g] = m_new;
                sh.l[g] = __fmaf_rn(sh.l[g], al, sum);
            }
        }
        named_bar_sync(1, ATTN_THREADS);

        // ---- P.V ------------------------------------------------------------
#pragma unroll
        for (int g = 0; g < GP; g++) {
            const float al = g < G ? sh.alpha[g] : 0.f;
#pragma unroll
            for (int e = 0; e < E; e++) acc[g][e] *= al;
        }
#pragma unroll
        for (int k = 0; k < DEC_TPW; k++) {
            const int t = warp + 8 * k;
            if (t >= n) break;                          // uniform over the warp
            float vf[E];
            dec_load<E, H>(Vs + ((size_t)t * hd + E * lane) * KB, vf);
            float p[GP];
            if constexpr (GP >= 4) {
#pragma unroll
                for (int g4 = 0; g4 < GP; g4 += 4) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(Pt + t * GP + g4);
                    p[g4] = p4.x; p[g4 + 1] = p4.y; p[g4 + 2] = p4.z; p[g4 + 3] = p4.w;
                }
            } else {
#pragma unroll
                for (int g = 0; g < GP; g++) p[g] = Pt[t * GP + g];
            }
#pragma unroll
            for (int g = 0; g < GP; g++)
#pragma unroll
                for (int e = 0; e < E; e++) acc[g][e] = __fmaf_rn(p[g], vf[e], acc[g][e]);
        }
        named_bar_sync(1, ATTN_THREADS);                // stage st and the score tiles are free again

        if (tid == 0 && issued < nsub) {
            // order this CTA's generic reads of the stage before the async copy into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (dec_issue<E, H>(a, pt, c0, ntok, issued, ring + (size_t)(issued % stages) * stage_bytes,
                                &bars[issued % stages]))
                issued++;
            else
                sh.fail = 1;
        }
    }
    if (j < nsub) {
        // abandoned (fault word set): no copy of this CTA may still be landing
        // in its shared memory when it exits
        if (tid == 0)
            for (int s = j; s < issued; s++) mbar_wait(&bars[s % stages], (uint32_t)((s / stages) & 1), nullptr, 0);
        return;
    }

    // ---- the chunk's partial: warp sums meet in shared memory ------------------
    float *red = reinterpret_cast<float *>(ring);       // [warp][GP][hd]; every copy has landed
#pragma unroll
    for (int g = 0; g < GP; g++)
#pragma unroll
        for (int e = 0; e < E; e++) red[((size_t)warp * GP + g) * hd + E * lane + e] = acc[g][e];
    named_bar_sync(1, ATTN_THREADS);
    for (int i = tid; i < G * hd; i += ATTN_THREADS) {
        const int g = i / hd, d = i % hd;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < ATTN_WARPS; w++) s += red[((size_t)w * GP + g) * hd + d];
        float *pp = a.part + (((long long)col * a.n_heads + hk * G + g) * a.n_splits + chunk) * (hd + 2);
        pp[d] = s;
        if (d == 0) { pp[hd] = sh.m[g]; pp[hd + 1] = sh.l[g]; }
    }
    __threadfence();
    named_bar_sync(1, ATTN_THREADS);
    __shared__ int last;
    if (tid == 0) last = atomicAdd(&a.counters[col * a.n_kv + hk], 1) == n_active - 1;
    named_bar_sync(1, ATTN_THREADS);
    if (!last) return;
    __threadfence();
    // last CTA of (column, kv head): merge the chunks in order
    for (int i = tid; i < G * hd; i += ATTN_THREADS) {
        const int g = i / hd, d = i % hd;
        const float *base = a.part + ((long long)col * a.n_heads + hk * G + g) * a.n_splits * (hd + 2);
        float M = -INFINITY;
        for (int c = 0; c < n_active; c++) M = fmaxf(M, __ldcg(base + c * (hd + 2) + hd));
        float L = 0.f, A = 0.f;
        for (int c = 0; c < n_active; c++) {
            const float *pp = base + c * (hd + 2);
            const float f = expf(__ldcg(pp + hd) - M);
            L = __fmaf_rn(__ldcg(pp + hd + 1), f, L);
            A = __fmaf_rn(__ldcg(pp + d), f, A);
        }
        a.out[(long long)col * a.out_ld + (long long)(hk * G + g) * hd + d] = A / L;
    }
    if (tid == 0) a.counters[col * a.n_kv + hk] = 0;
}
