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

// Values E*lane .. E*lane+E-1 of row t (context position pos) of a
// shared-memory K or V tile as floats (f16 rows are chunk-swizzled, kv_swz).
template <int E, bool H>
__device__ __forceinline__ void dec_load(const unsigned char *tile, int t, int pos, int lane, float (&f)[E]) {
    constexpr int hd = 32 * E;
    const unsigned char *p =
        H ? tile + ((size_t)t * hd + kv_swz(pos, E * lane, hd)) * 2 : tile + ((size_t)t * hd + E * lane) * 4;
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
    const long long head_off = (long long)blockIdx.y * 2 * P * hd;    // the kv head's K block in the page
    const long long v_off = (long long)P * hd;
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
            dec_load<E, H>(Ks, warp + 8 * k, c0 + j * DEC_SUB + warp + 8 * k, lane, kf);
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
            dec_load<E, H>(Vs, t, c0 + j * DEC_SUB + t, lane, vf);
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

// ---------------------------------------------------------------------------
// Persistent tensor-core decode attention, for wide steps (16 or more
// columns, where the step's weight products also run on f16 tensor cores)
// over an f16 pool.
//
// One CTA per SM runs until the step's work is gone.  A work item is (chunk
// of at most CH context tokens, kv head) of one column; the host orders the
// columns by context length, longest first (a.order), picks CH so that there
// are several items per SM (a.attn_chunk), and gives the prefix sums of the
// columns' chunk counts (a.chunk_pfx): item i is chunk i / n_kv of that
// list, kv head i % n_kv.  The producer lane (warp 8) takes items from a
// per-layer counter (atomicAdd: long items start first, short ones fill the
// gaps) and streams their 64-token sub-tiles into the ring without a break
// between items.  A stage carries its own description (column, head, chunk,
// tokens, first / last flags); the first stage of an item also the item's G
// query rows (f32, one more bulk copy).
//
// Consumer warp w takes tokens 8w .. 8w+7 of every sub-tile:
//   S (16 x 8)  = Q (16 x hd) . K^T        mma.m16n8k16, f16 in, f32 out
//                 (rows: the G query heads of the kv head, zero past G)
//   online softmax per row over the 8 tokens (4 lanes hold a row)
//   O (16 x hd) += P (16 x 8) . V (8 x hd)  mma.m16n8k8; the accumulator
//                 fragment of S is P's operand fragment (f16 pairs)
// K and V fragments come from ldmatrix, free of bank conflicts because the
// pool's rows are chunk-swizzled by position (kv_swz).  Queries and
// probabilities enter the products rounded to f16, as the wide steps'
// activations do.  At the end of an item the warps' softmax states and
// accumulators meet in shared memory; the item's output is written directly
// when it is its column's only chunk, else as a partial that the last warp
// to finish the column merges in chunk order.  Every CTA-level wait here is
// a bounded mbarrier wait (no named barrier): a wait that runs out sets the
// fault word and the CTA winds down without leaving a copy in flight.  The
// last consumer warp of the grid to exit resets the layer's work counters,
// so the launch can be replayed.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void *p, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ uint32_t h2_bits(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

struct PersMeta {
    int col, hk, chunk, n;      // item and tokens in this sub-tile
    int c0, flags, pos, pad;    // chunk start, PM_* flags, the column's position
};
enum : int { PM_FIRST = 1, PM_LAST = 2, PM_END = 4 };
#define PERS_STAGES_MAX 8
#define PERS_THREADS (ATTN_THREADS + 32)   // 8 consumer warps + 1 producer warp

__host__ __device__ inline size_t pers_stage_bytes(int hd) {
    return (size_t)2 * DEC_SUB * hd * 2 + (size_t)ATTN_MAX_G * hd * 4;   // K, V (f16) + query rows (f32)
}
__host__ __device__ inline size_t pers_pfx_bytes(int max_cols) { return (((size_t)max_cols + 1) * 4 + 15) / 16 * 16; }
#define PERS_MAX_ITEM_PAGES 1024   // pages of one work item (the host caps the chunk accordingly)

__host__ __device__ inline size_t pers_fixed_bytes(int hd, int max_cols) {
    return (size_t)ATTN_WARPS * ATTN_MAX_G * (hd + 2) * 4        // warp states
           + (size_t)PERS_MAX_ITEM_PAGES * 4                     // the current item's page list
           + pers_pfx_bytes(max_cols)                            // chunk prefix sums
           + (size_t)PERS_STAGES_MAX * sizeof(PersMeta) + 16     // stage descriptions, flag
           + (size_t)(2 * PERS_STAGES_MAX + 2) * 8;               // full / empty / combine mbarriers
}
// Stages that fit beside the fixed part in `budget` bytes (0 .. PERS_STAGES_MAX).
__host__ __device__ inline int pers_stages(int hd, int max_cols, size_t budget) {
    const size_t fx = pers_fixed_bytes(hd, max_cols);
    const int s = budget > fx ? (int)((budget - fx) / pers_stage_bytes(hd)) : 0;
    return s > PERS_STAGES_MAX ? PERS_STAGES_MAX : s;
}

template <int E>
__global__ void __launch_bounds__(PERS_THREADS, 1) k_attn_pers(AttnArgs a, int stages, int max_cols) {
    constexpr int hd = 32 * E, NB = hd / 8, KS = hd / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3, r8 = lane & 7, m4 = lane >> 3;
    const int G = a.n_heads / a.n_kv, nkv = a.n_kv;
    const size_t sb = pers_stage_bytes(hd), kvb = (size_t)2 * DEC_SUB * hd * 2;

    unsigned char *ring = cmolcu_smem;
    float *red = reinterpret_cast<float *>(ring + (size_t)stages * sb);                 // [8][8][hd + 2]
    int *pages = reinterpret_cast<int *>(red + (size_t)ATTN_WARPS * ATTN_MAX_G * (hd + 2));   // [1024]
    int *pfx = pages + PERS_MAX_ITEM_PAGES;
    PersMeta *meta = reinterpret_cast<PersMeta *>(reinterpret_cast<unsigned char *>(pfx) + pers_pfx_bytes(max_cols));
    int *fail = reinterpret_cast<int *>(meta + PERS_STAGES_MAX);
    uint64_t *full = reinterpret_cast<uint64_t *>(fail + 4);
    uint64_t *empty = full + PERS_STAGES_MAX;
    uint64_t *comb_full = empty + PERS_STAGES_MAX, *comb_empty = comb_full + 1;
    volatile int *vfail = fail;

    pdl_wait();
    const int nlive = *a.attn_n;
    const int CH = *a.attn_chunk;
    for (int i = tid; i <= nlive; i += PERS_THREADS) pfx[i] = a.chunk_pfx[i];
    if (tid == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ATTN_WARPS);
        }
        mbar_init(comb_full, ATTN_WARPS);
        mbar_init(comb_empty, ATTN_WARPS);
        fence_mbar_init();
        *fail = 0;
    }
    __syncthreads();
    const int total = pfx[nlive] * nkv;
    int *work = a.work + 2 * a.layer;                   // [0] next item, [1] consumer warps done

    if (warp == ATTN_WARPS) {
        // ---- producer warp ----------------------------------------------------------
        // All 32 lanes load an item's description and page list (into
        // shared memory, one parallel round); lane 0 issues the copies.  The
        // next item's index is taken while the current one streams.
        if (lane == 0) fence_proxy_async_global();      // K, V and q of this step came through the generic proxy
        const int P = a.page_tokens;
        int k = 0;                                      // stages issued so far (lane 0's count, broadcast)
        bool bad = false;
        int nxt = 0;
        if (lane == 0) nxt = *vfail ? total : atomicAdd(&work[0], 1);
        nxt = __shfl_sync(0xffffffffu, nxt, 0);
        while (nxt < total) {
            const int i = nxt;
            const int u = i / nkv, hk = i % nkv;
            int lo = 0, hi = nlive - 1;                 // column rank: the last r with pfx[r] <= u
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (pfx[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const int col = a.order[lo], chunk = u - pfx[lo];
            const int pos = a.pos[col];
            const int srow = a.slot ? a.slot[col] : col;
            const int c0 = chunk * CH, ntok = min(CH, pos + 1 - c0), nsub = (ntok + DEC_SUB - 1) / DEC_SUB;
            const int npg_item = (ntok + P - 1) / P;    // c0 is a multiple of P (CH is)
            const int *pt = a.page_table + (long long)srow * a.max_pages + c0 / P;
            bool lbad = npg_item > PERS_MAX_ITEM_PAGES;
            for (int p = lane; p < npg_item && !lbad; p += 32) {
                const int pg = pt[p];
                if (pg < 0 || pg >= a.n_pages) lbad = true;
                pages[p] = pg;
            }
            if (__any_sync(0xffffffffu, lbad)) {
                if (lane == 0 && a.fault) atomicExch(a.fault, FAULT_BAD_PAGE);
                bad = true;
                break;
            }
            __syncwarp();
            if (lane == 0) {
                nxt = *vfail ? total : atomicAdd(&work[0], 1);   // in flight while this item streams
                const uint32_t blk = (uint32_t)(P * hd * 2);
                const long long head_off = (long long)hk * 2 * P * hd;
                const long long v_off = (long long)P * hd;
                const unsigned char *pool = static_cast<const unsigned char *>(a.kv_pages);
                for (int j = 0; j < nsub; j++, k++) {
                    const int st = k % stages;
                    if (k >= stages &&
                        !mbar_wait(&empty[st], (uint32_t)(((k / stages) - 1) & 1), a.fault, FAULT_ATTN_WAIT)) {
                        bad = true;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    const int n = min(DEC_SUB, ntok - j * DEC_SUB), npg = (n + P - 1) / P;
                    const int pg0 = j * (DEC_SUB / P);
                    unsigned char *stage = ring + (size_t)st * sb;
                    PersMeta &md = meta[st];
                    md.col = col; md.hk = hk; md.chunk = chunk; md.n = n; md.c0 = c0; md.pos = pos;
                    md.flags = (j == 0 ? PM_FIRST : 0) | (j == nsub - 1 ? PM_LAST : 0);
                    const uint32_t qbytes = j == 0 ? (uint32_t)(G * hd * 4) : 0u;
                    mbar_arrive_expect_tx(&full[st], 2u * npg * blk + qbytes);
                    for (int p = 0; p < npg; p++) {
                        const unsigned char *kp = pool + ((long long)pages[pg0 + p] * a.page_elems + head_off) * 2;
                        bulk_g2s(stage + (size_t)p * blk, kp, blk, &full[st]);
                        bulk_g2s(stage + (size_t)DEC_SUB * hd * 2 + (size_t)p * blk, kp + v_off * 2, blk, &full[st]);
                    }
                    if (qbytes)
                        bulk_g2s(stage + kvb, a.q + (long long)col * a.q_ld + (long long)hk * G * hd, qbytes,
                                 &full[st]);
                }
            }
            nxt = __shfl_sync(0xffffffffu, nxt, 0);
            bad = __shfl_sync(0xffffffffu, bad ? 1 : 0, 0) != 0;
            __syncwarp();                               // the page list is reused by the next item
            if (bad) break;
        }
        if (lane != 0) return;
        // the end marker (after a failure too): one more stage, no data
        const int st = k % stages;
        bool can = true;
        if (k >= stages) can = mbar_wait(&empty[st], (uint32_t)(((k / stages) - 1) & 1), a.fault, FAULT_ATTN_WAIT);
        if (bad || !can) *vfail = 1;
        if (can) {
            meta[st].flags = PM_END;
            mbar_arrive(&full[st]);
        }
        // every copy issued lands before this thread exits.  Sub-tile k -
        // stages shares the end marker's stage: when the marker went in, the
        // consumers had released that stage, so its copy has landed (and its
        // barrier has moved one phase further: waiting on it would not end).
        for (int s = k - 1; s >= 0 && s >= k - stages + (can ? 1 : 0); s--)
            mbar_wait(&full[s % stages], (uint32_t)((s / stages) & 1), nullptr, 0);
        return;
    }

    // ---- consumers ------------------------------------------------------------------
    uint32_t qa[KS][4];
    float acc[NB][4];
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};   // rows gq and gq + 8
#pragma unroll
    for (int ks = 0; ks < KS; ks++) qa[ks][0] = qa[ks][1] = qa[ks][2] = qa[ks][3] = 0u;
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
    int items = 0;                                      // items this CTA has combined
    const int row0 = 8 * warp;                          // this warp's rows of every sub-tile
    for (int k = 0;; k++) {
        const int st = k % stages;
        if (!mbar_wait(&full[st], (uint32_t)((k / stages) & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        const PersMeta md = meta[st];
        if (md.flags & PM_END) break;
        const unsigned char *Ks = ring + (size_t)st * sb;
        unsigned char *Vs = ring + (size_t)st * sb + (size_t)DEC_SUB * hd * 2;
        if (md.flags & PM_FIRST) {
            // query fragments (rows: the G heads, zero past G) from the f32 rows
            const float *qf = reinterpret_cast<const float *>(Ks + kvb);
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
                const int d0 = 16 * ks + 2 * tq;
                const float2 z = make_float2(0.f, 0.f);
                const float2 x0 = gq < G ? *reinterpret_cast<const float2 *>(qf + gq * hd + d0) : z;
                const float2 x2 = gq < G ? *reinterpret_cast<const float2 *>(qf + gq * hd + d0 + 8) : z;
                const float2 x1 = gq + 8 < G ? *reinterpret_cast<const float2 *>(qf + (gq + 8) * hd + d0) : z;
                const float2 x3 = gq + 8 < G ? *reinterpret_cast<const float2 *>(qf + (gq + 8) * hd + d0 + 8) : z;
                qa[ks][0] = h2_bits(x0.x, x0.y);
                qa[ks][1] = h2_bits(x1.x, x1.y);
                qa[ks][2] = h2_bits(x2.x, x2.y);
                qa[ks][3] = h2_bits(x3.x, x3.y);
            }
#pragma unroll
            for (int b = 0; b < NB; b++) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
            m_run[0] = m_run[1] = -INFINITY;
            l_run[0] = l_run[1] = 0.f;
        }
        const int n = md.n;
        if (n < row0 + 8) {
            // rows past the context hold stale or never-written values: zero
            // this warp's V rows there (probability 0 must not meet a NaN)
            for (int i = lane; i < hd; i += 32) {
                const int r = i / (hd / 8);
                if (row0 + r >= n)
                    reinterpret_cast<uint4 *>(Vs + (size_t)(row0 + r) * hd * 2)[i % (hd / 8)] = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        // ---- S = Q K^T for the warp's 8 tokens -----------------------------------------
        float S[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < hd / 32; kk++) {
            uint32_t k0, k1, k2, k3;                    // K chunks 4kk .. 4kk+3 of the 8 rows
            ldsm_x4(Ks + ((size_t)(row0 + r8) * hd + (((4 * kk + m4) ^ r8) << 3)) * 2, k0, k1, k2, k3);
            mma_16816(S, qa[2 * kk][0], qa[2 * kk][1], qa[2 * kk][2], qa[2 * kk][3], k0, k1);
            mma_16816(S, qa[2 * kk + 1][0], qa[2 * kk + 1][1], qa[2 * kk + 1][2], qa[2 * kk + 1][3], k2, k3);
        }
        // ---- online softmax: row gq (S[0], S[1]), row gq + 8 (S[2], S[3]) -------------
        const bool v0 = row0 + 2 * tq < n, v1 = row0 + 2 * tq + 1 < n;
        float p[4], al[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float s0 = v0 ? S[2 * h] * a.scale : -INFINITY;
            const float s1 = v1 ? S[2 * h + 1] * a.scale : -INFINITY;
            float mx = fmaxf(s0, s1);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_run[h], mx);
            const float e0 = s0 == -INFINITY ? 0.f : expf(s0 - m_new);
            const float e1 = s1 == -INFINITY ? 0.f : expf(s1 - m_new);
            float sum = e0 + e1;
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            al[h] = m_run[h] == -INFINITY ? 0.f : expf(m_run[h] - m_new);
            l_run[h] = __fmaf_rn(l_run[h], al[h], sum);
            m_run[h] = m_new;
            p[2 * h] = e0;
            p[2 * h + 1] = e1;
        }
        if (__any_sync(0xffffffffu, al[0] != 1.f || al[1] != 1.f)) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                acc[b][0] *= al[0]; acc[b][1] *= al[0];
                acc[b][2] *= al[1]; acc[b][3] *= al[1];
            }
        }
        const uint32_t pa0 = h2_bits(p[0], p[1]), pa1 = h2_bits(p[2], p[3]);
        // ---- O += P V -------------------------------------------------------------------
#pragma unroll
        for (int nb = 0; nb < hd / 32; nb++) {
            uint32_t b0, b1, b2, b3;                    // V chunks 4nb .. 4nb+3 of the 8 rows, transposed
            ldsm_x4_t(Vs + ((size_t)(row0 + r8) * hd + (((4 * nb + m4) ^ r8) << 3)) * 2, b0, b1, b2, b3);
            mma_1688(acc[4 * nb + 0], pa0, pa1, b0);
            mma_1688(acc[4 * nb + 1], pa0, pa1, b1);
            mma_1688(acc[4 * nb + 2], pa0, pa1, b2);
            mma_1688(acc[4 * nb + 3], pa0, pa1, b3);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);         // the stage is free; its description is in md
        if (!(md.flags & PM_LAST)) continue;

        // ---- end of an item: combine the warps (comb_full counts the warps whose
        // states are in red, comb_empty those done reading it) ------------------------------
        const int col = md.col, hk = md.hk, chunk = md.chunk;
        if (items > 0 && !mbar_wait(comb_empty, (uint32_t)((items - 1) & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        if (gq < G) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float *r0 = red + ((size_t)warp * ATTN_MAX_G + gq) * (hd + 2) + 8 * b + 2 * tq;
                r0[0] = acc[b][0];
                r0[1] = acc[b][1];
            }
            if (tq == 0) {
                red[((size_t)warp * ATTN_MAX_G + gq) * (hd + 2) + hd] = m_run[0];
                red[((size_t)warp * ATTN_MAX_G + gq) * (hd + 2) + hd + 1] = l_run[0];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(comb_full);
        if (!mbar_wait(comb_full, (uint32_t)(items & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        const int n_active = md.pos / CH + 1;           // chunks of this column
        for (int i = tid; i < G * hd; i += ATTN_THREADS) {
            const int g = i / hd, d = i % hd;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < ATTN_WARPS; w++) M = fmaxf(M, red[((size_t)w * ATTN_MAX_G + g) * (hd + 2) + hd]);
            float L = 0.f, A = 0.f;
#pragma unroll
            for (int w = 0; w < ATTN_WARPS; w++) {
                const float *rw = red + ((size_t)w * ATTN_MAX_G + g) * (hd + 2);
                const float mw = rw[hd];
                const float f = mw == -INFINITY ? 0.f : expf(mw - M);
                L = __fmaf_rn(rw[hd + 1], f, L);
                A = __fmaf_rn(rw[d], f, A);
            }
            if (n_active == 1) {
                a.out[(long long)col * a.out_ld + (long long)(hk * G + g) * hd + d] = A / L;
            } else {
                float *pp = a.part + (((long long)col * a.n_heads + hk * G + g) * a.n_splits + chunk) * (hd + 2);
                pp[d] = A;
                if (d == 0) { pp[hd] = M; pp[hd + 1] = L; }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(comb_empty);         // this warp is done reading red
        items++;
        if (n_active > 1) {
            // every warp counts its share of the partial; the warp that
            // completes the column's count (all chunks, all warps) merges it
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(&a.counters[col * nkv + hk], 1) == n_active * ATTN_WARPS - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                for (int i = lane; i < G * hd; i += 32) {
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
                if (lane == 0) a.counters[col * nkv + hk] = 0;
            }
        }
    }
    // each consumer warp counts its exit; the last one of the grid resets the
    // layer's work counters (every producer has taken its last item by then)
    if (lane == 0 && atomicAdd(&work[1], 1) == (int)gridDim.x * ATTN_WARPS - 1) {
        work[0] = 0;
        work[1] = 0;
    }
}
