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
// list, kv head i % n_kv.  Each CTA copies the column table (column,
// position, slot by rank) into shared memory before the previous kernel of
// the step has finished.  Four roles share the CTA (warps):
//   item warp (9)    takes items from a per-layer counter (atomicAdd: long
//                    items start first, short ones fill the gaps) one item
//                    ahead, decodes them and copies their page lists into
//                    two item slots;
//   producer (8)     one lane that streams each item's 64-token sub-tiles
//                    into the ring.  It touches only shared memory, barriers
//                    and bulk copies, so its barrier releases never wait on
//                    an atomic or a global load in flight, and consecutive
//                    items follow each other without a break;
//   consumers (0-7)  the products and the softmax, below;
//   merge warp (10)  counts each partial this CTA wrote on its column's
//                    counter; the CTA that completes the count merges the
//                    column's chunks, while the consumers carry on.
// A stage carries its own description (column, head, chunk, tokens, first /
// last flags); the first stage of an item also the item's G query rows (f32,
// one more bulk copy).
//
// Consumer warp w takes tokens 8w .. 8w+7 of every sub-tile.  It copies its
// K and V fragments into registers (ldmatrix, free of bank conflicts because
// the pool's rows are chunk-swizzled by position, kv_swz) and releases the
// stage at once; the products and the softmax run from registers while the
// ring refills:
//   S (16 x 8)  = Q (16 x hd) . K^T        mma.m16n8k16, f16 in, f32 out
//                 (rows: the G query heads of the kv head, zero past G)
//   online softmax per row over the 8 tokens (4 lanes hold a row)
//   O (16 x hd) += P (16 x 8) . V (8 x hd)  mma.m16n8k8; the accumulator
//                 fragment of S is P's operand fragment (f16 pairs)
// The queries enter the product pre-multiplied by scale * log2(e) and
// rounded to f16 (as the wide steps' activations are), so scores are in
// base-2 units and the weights are exp2(s - m).  The reference maximum m of
// a row moves only when a score passes it by more than PERS_SLACK (weights
// stay <= 2^PERS_SLACK, well inside f16), so the accumulator is rarely
// rescaled; each lane sums its own weights and the four lanes of a row add
// their sums once, at the end of the item.  At the end of an item the warps'
// softmax states and accumulators meet in shared memory; the item's output
// is written directly when it is its column's only chunk, else as a partial
// for the merge warps (chunk order).  Every
// CTA-level wait here is a bounded mbarrier wait (no named barrier): a wait
// that runs out sets the fault word and the CTA winds down without leaving a
// copy in flight.  The last consumer warp of the grid to exit resets the
// layer's work counters, so the launch can be replayed.
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
// One work item as the item warp hands it to the producer.
struct PersItem {
    int col, hk, chunk, pos;
    int c0, ntok, npg, end;     // chunk start, tokens, pages; end: no more items
};
#define PERS_STAGES_MAX 8
#define PERS_THREADS (ATTN_THREADS + 96)   // 8 consumer warps, producer, item and merge warps
#define PERS_MAX_ITEM_PAGES 256            // pages of one work item (the host caps the chunk accordingly)
#define PERS_MQ 4                          // merge queue entries
#define PERS_SLACK 8.f                     // base-2 headroom of the softmax reference maximum

__host__ __device__ inline size_t pers_stage_bytes(int hd, int G) {
    return (size_t)2 * DEC_SUB * hd * 2 + (size_t)G * hd * 4;   // K, V (f16) + the item's query rows (f32)
}
__host__ __device__ inline size_t pers_cols_bytes(int max_cols) { return ((size_t)max_cols * 4 + 15) / 16 * 16; }
__host__ __device__ inline size_t pers_pfx_bytes(int max_cols) { return pers_cols_bytes(max_cols + 1); }
#define PERS_BARRIERS (2 * PERS_STAGES_MAX + 2 + 4 + 2 * PERS_MQ)

__host__ __device__ inline size_t pers_fixed_bytes(int hd, int G, int max_cols) {
    return (size_t)ATTN_WARPS * G * (hd + 2) * 4                 // warp states
           + (size_t)2 * PERS_MAX_ITEM_PAGES * 4                 // item slots' page lists
           + pers_pfx_bytes(max_cols)                            // chunk prefix sums
           + 3 * pers_cols_bytes(max_cols)                       // column, position, slot by rank
           + (size_t)PERS_STAGES_MAX * sizeof(PersMeta)          // stage descriptions
           + 2 * sizeof(PersItem) + PERS_MQ * 16 + 16            // item slots, merge queue, flag
           + (size_t)PERS_BARRIERS * 8;
}
// Stages that fit beside the fixed part in `budget` bytes (0 .. PERS_STAGES_MAX).
__host__ __device__ inline int pers_stages(int hd, int G, int max_cols, size_t budget) {
    const size_t fx = pers_fixed_bytes(hd, G, max_cols);
    const int s = budget > fx ? (int)((budget - fx) / pers_stage_bytes(hd, G)) : 0;
    return s > PERS_STAGES_MAX ? PERS_STAGES_MAX : s;
}

// 4-byte asynchronous global -> shared copy (completion: cp_async_wait_all).
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bounded wait that also gives up as soon as another role has failed.
__device__ __forceinline__ bool pers_wait(uint64_t *bar, uint32_t parity, volatile int *vfail, unsigned int *fault) {
    for (uint32_t i = 0; i < CMOLCU_SPIN_LIMIT; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*vfail) return false;
    }
    if (fault) atomicExch(fault, FAULT_ATTN_WAIT);
    return false;
}

// Decode item i from the shared column table and start the copy of its page
// list into `pages` (every lane of the warp calls this; the caller waits).
__device__ __forceinline__ PersItem pers_item(const AttnArgs &a, int i, int nkv, int nlive, int CH,
                                              const int *pfx, const int *t_col, const int *t_pos,
                                              const int *t_srow, int *pages, int lane) {
    const int u = i / nkv;
    int lo = 0, hi = nlive - 1;                         // column rank: the last r with pfx[r] <= u
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pfx[mid] <= u) lo = mid; else hi = mid - 1;
    }
    PersItem it;
    it.col = t_col[lo];
    it.hk = i % nkv;
    it.chunk = u - pfx[lo];
    it.pos = t_pos[lo];
    it.c0 = it.chunk * CH;
    it.ntok = min(CH, it.pos + 1 - it.c0);
    const int P = a.page_tokens;
    it.npg = (it.ntok + P - 1) / P;                     // c0 is a multiple of P (CH is)
    it.end = 0;
    const int *pt = a.page_table + (long long)t_srow[lo] * a.max_pages + it.c0 / P;
    if (it.npg <= PERS_MAX_ITEM_PAGES)
        for (int p = lane; p < it.npg; p += 32) cp_async4(pages + p, pt + p);
    return it;
}

// After the page-list copy has landed (wait + __syncwarp): every entry a
// valid page of the pool (warp-uniform answer).
__device__ __forceinline__ bool pers_pages_ok(const AttnArgs &a, const PersItem &it, const int *pages, int lane) {
    bool bad = it.npg > PERS_MAX_ITEM_PAGES;
    for (int p = lane; p < it.npg && !bad; p += 32) {
        const int pg = pages[p];
        bad = pg < 0 || pg >= a.n_pages;
    }
    return !__any_sync(0xffffffffu, bad);
}

template <int E>
__global__ void __launch_bounds__(PERS_THREADS, 1) k_attn_pers(AttnArgs a, int stages, int max_cols) {
    constexpr int hd = 32 * E, NB = hd / 8, KS = hd / 16, KQ = hd / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3, r8 = lane & 7, m4 = lane >> 3;
    const int G = a.n_heads / a.n_kv, nkv = a.n_kv;
    const size_t sb = pers_stage_bytes(hd, G), kvb = (size_t)2 * DEC_SUB * hd * 2;

    unsigned char *ring = cmolcu_smem;
    float *red = reinterpret_cast<float *>(ring + (size_t)stages * sb);                 // [8][G][hd + 2]
    int *ipages = reinterpret_cast<int *>(red + (size_t)ATTN_WARPS * G * (hd + 2));     // [2][256]
    int *pfx = ipages + 2 * PERS_MAX_ITEM_PAGES;
    int *t_col = reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(pfx) + pers_pfx_bytes(max_cols));
    int *t_pos = reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(t_col) + pers_cols_bytes(max_cols));
    int *t_srow = reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(t_pos) + pers_cols_bytes(max_cols));
    PersMeta *meta = reinterpret_cast<PersMeta *>(reinterpret_cast<unsigned char *>(t_srow) + pers_cols_bytes(max_cols));
    PersItem *idesc = reinterpret_cast<PersItem *>(meta + PERS_STAGES_MAX);            // [2]
    int4 *mq = reinterpret_cast<int4 *>(idesc + 2);                                      // [PERS_MQ]
    int *fail = reinterpret_cast<int *>(mq + PERS_MQ);
    uint64_t *full = reinterpret_cast<uint64_t *>(fail + 4);
    uint64_t *empty = full + PERS_STAGES_MAX;
    uint64_t *comb_full = empty + PERS_STAGES_MAX, *comb_empty = comb_full + 1;
    uint64_t *it_full = comb_empty + 1, *it_empty = it_full + 2;
    uint64_t *mq_full = it_empty + 2, *mq_empty = mq_full + PERS_MQ;
    volatile int *vfail = fail;

    // The step's column table was uploaded before the step's first kernel:
    // read it while the previous kernel finishes.
    const int nlive = *a.attn_n;
    const int CH = *a.attn_chunk;
    for (int i = tid; i <= nlive; i += PERS_THREADS) pfx[i] = a.chunk_pfx[i];
    for (int i = tid; i < nlive; i += PERS_THREADS) {
        const int col = a.order[i];
        t_col[i] = col;
        t_pos[i] = a.pos[col];
        t_srow[i] = a.slot ? a.slot[col] : col;
    }
    if (tid == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ATTN_WARPS);
        }
        mbar_init(comb_full, ATTN_WARPS);
        mbar_init(comb_empty, ATTN_WARPS);
        for (int s = 0; s < 2; s++) {
            mbar_init(&it_full[s], 1);
            mbar_init(&it_empty[s], 1);
        }
        for (int s = 0; s < PERS_MQ; s++) {
            mbar_init(&mq_full[s], ATTN_WARPS);
            mbar_init(&mq_empty[s], 1);
        }
        fence_mbar_init();
        *fail = 0;
    }
    pdl_wait();
    __syncthreads();
    const int total = pfx[nlive] * nkv;
    int *work = a.work + 2 * a.layer;                   // [0] next item, [1] consumer warps done

    if (warp == ATTN_WARPS + 1) {
        // ---- item warp: takes items from the layer's counter one ahead of the
        // producer, decodes them and copies their page lists into the two item
        // slots.  Its global reads and atomics keep the producer's releases
        // free of outstanding memory operations.
        for (int j = 0;; j++) {
            const int sl = j & 1;
            int ok = 1;
            if (lane == 0 && j >= 2) ok = pers_wait(&it_empty[sl], (uint32_t)(((j >> 1) - 1) & 1), vfail, a.fault);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            int i = total;
            if (lane == 0 && !*vfail) i = atomicAdd(&work[0], 1);
            i = __shfl_sync(0xffffffffu, i, 0);
            int *pl = ipages + sl * PERS_MAX_ITEM_PAGES;
            PersItem it{};
            bool good = true;
            if (i < total) {
                it = pers_item(a, i, nkv, nlive, CH, pfx, t_col, t_pos, t_srow, pl, lane);
                cp_async_wait_all();
                __syncwarp();
                good = pers_pages_ok(a, it, pl, lane);
            }
            if (lane == 0) {
                if (!good && a.fault) atomicExch(a.fault, FAULT_BAD_PAGE);
                if (!good) *vfail = 1;
                it.end = i >= total || !good;
                idesc[sl] = it;
                mbar_arrive(&it_full[sl]);
            }
            if (i >= total || !good) break;
        }
        return;
    }

    if (warp == ATTN_WARPS + 2) {
        // ---- merge warp: for each item of this CTA that wrote a partial, count
        // it on the column's counter; the CTA that completes the count merges
        // the column's chunks in chunk order.
        for (int j = 0;; j++) {
            const int q = j % PERS_MQ;
            int ok = 1;
            if (lane == 0) ok = pers_wait(&mq_full[q], (uint32_t)((j / PERS_MQ) & 1), vfail, a.fault);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const int4 e = mq[q];                       // col, kv head, chunks; w = 1: no more entries
            __syncwarp();
            if (lane == 0) mbar_arrive(&mq_empty[q]);
            if (e.w) break;
            const int col = e.x, hk = e.y, n_active = e.z;
            __threadfence();                            // the consumers' partial stores, before the count
            int last = 0;
            if (lane == 0) last = atomicAdd(&a.counters[col * nkv + hk], 1) == n_active - 1;
            if (!__shfl_sync(0xffffffffu, last, 0)) continue;
            __threadfence();
            for (int g = 0; g < G; g++) {
                const float *base = a.part + ((long long)col * a.n_heads + hk * G + g) * a.n_splits * (hd + 2);
                float M = -INFINITY;
                for (int c = 0; c < n_active; c++) M = fmaxf(M, __ldcg(base + c * (hd + 2) + hd));
                float L = 0.f, A[KQ];
#pragma unroll
                for (int t = 0; t < KQ; t++) A[t] = 0.f;
                for (int c = 0; c < n_active; c++) {
                    const float *pp = base + c * (hd + 2);
                    const float f = exp2f(__ldcg(pp + hd) - M);
                    L = __fmaf_rn(__ldcg(pp + hd + 1), f, L);
#pragma unroll
                    for (int t = 0; t < KQ; t++) A[t] = __fmaf_rn(__ldcg(pp + lane + 32 * t), f, A[t]);
                }
#pragma unroll
                for (int t = 0; t < KQ; t++)
                    a.out[(long long)col * a.out_ld + (long long)(hk * G + g) * hd + lane + 32 * t] = A[t] / L;
            }
            if (lane == 0) a.counters[col * nkv + hk] = 0;
        }
        return;
    }

    if (warp == ATTN_WARPS) {
        // ---- producer lane: streams each item's 64-token sub-tiles into the
        // ring (shared-memory reads, barrier operations and bulk copies only)
        if (lane != 0) return;
        fence_proxy_async_global();                     // K, V and q of this step came through the generic proxy
        const int P = a.page_tokens;
        const uint32_t blk = (uint32_t)(P * hd * 2);
        const long long v_off = (long long)P * hd;
        const unsigned char *pool = static_cast<const unsigned char *>(a.kv_pages);
        int k = 0;                                      // stages issued so far
        bool bad = false;
        for (int j = 0; !bad; j++) {
            const int sl = j & 1;
            if (!pers_wait(&it_full[sl], (uint32_t)((j >> 1) & 1), vfail, a.fault)) {
                bad = true;
                break;
            }
            const PersItem it = idesc[sl];
            const int *pl = ipages + sl * PERS_MAX_ITEM_PAGES;
            if (it.end) break;
            const long long head_off = (long long)it.hk * 2 * P * hd;
            const int nsub = (it.ntok + DEC_SUB - 1) / DEC_SUB;
            for (int s = 0; s < nsub; s++, k++) {
                const int st = k % stages;
                if (k >= stages &&
                    !mbar_wait(&empty[st], (uint32_t)(((k / stages) - 1) & 1), a.fault, FAULT_ATTN_WAIT)) {
                    bad = true;
                    break;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                const int n = min(DEC_SUB, it.ntok - s * DEC_SUB), npg = (n + P - 1) / P;
                const int pg0 = s * (DEC_SUB / P);
                unsigned char *stage = ring + (size_t)st * sb;
                PersMeta &md = meta[st];
                md.col = it.col; md.hk = it.hk; md.chunk = it.chunk; md.n = n; md.c0 = it.c0; md.pos = it.pos;
                md.flags = (s == 0 ? PM_FIRST : 0) | (s == nsub - 1 ? PM_LAST : 0);
                const uint32_t qbytes = s == 0 ? (uint32_t)(G * hd * 4) : 0u;
                mbar_arrive_expect_tx(&full[st], 2u * npg * blk + qbytes);
                for (int p = 0; p < npg; p++) {
                    const unsigned char *kp = pool + ((long long)pl[pg0 + p] * a.page_elems + head_off) * 2;
                    bulk_g2s(stage + (size_t)p * blk, kp, blk, &full[st]);
                    bulk_g2s(stage + (size_t)DEC_SUB * hd * 2 + (size_t)p * blk, kp + v_off * 2, blk, &full[st]);
                }
                if (qbytes)
                    bulk_g2s(stage + kvb, a.q + (long long)it.col * a.q_ld + (long long)it.hk * G * hd, qbytes,
                             &full[st]);
            }
            mbar_arrive(&it_empty[sl]);                 // the slot's page list is no longer read
        }
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
    float m_run[2] = {-INFINITY, -INFINITY};            // reference maxima of rows gq and gq + 8 (base 2)
    float l_run[2] = {0.f, 0.f};                        // this lane's share of the rows' weight sums
    const float qscale = a.scale * 1.4426950408889634f;
#pragma unroll
    for (int ks = 0; ks < KS; ks++) qa[ks][0] = qa[ks][1] = qa[ks][2] = qa[ks][3] = 0u;
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
    int items = 0;                                      // items this CTA has combined
    int parts = 0;                                      // of them, the ones that wrote a partial
    bool ended = false;
    const int row0 = 8 * warp;                          // this warp's rows of every sub-tile
    for (int k = 0;; k++) {
        const int st = k % stages;
        if (!mbar_wait(&full[st], (uint32_t)((k / stages) & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        const PersMeta md = meta[st];
        if (md.flags & PM_END) {
            ended = true;
            break;
        }
        const unsigned char *Ks = ring + (size_t)st * sb;
        const unsigned char *Vs = Ks + (size_t)DEC_SUB * hd * 2;
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
                qa[ks][0] = h2_bits(x0.x * qscale, x0.y * qscale);
                qa[ks][1] = h2_bits(x1.x * qscale, x1.y * qscale);
                qa[ks][2] = h2_bits(x2.x * qscale, x2.y * qscale);
                qa[ks][3] = h2_bits(x3.x * qscale, x3.y * qscale);
            }
#pragma unroll
            for (int b = 0; b < NB; b++) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
            m_run[0] = m_run[1] = -INFINITY;
            l_run[0] = l_run[1] = 0.f;
        }
        // ---- the warp's K and V fragments into registers; the stage is released
        uint32_t kf[KQ][4], vf[KQ][4];                  // chunks 4c .. 4c+3 of the warp's 8 rows
#pragma unroll
        for (int c = 0; c < KQ; c++)
            ldsm_x4(Ks + ((size_t)(row0 + r8) * hd + (((4 * c + m4) ^ r8) << 3)) * 2, kf[c][0], kf[c][1], kf[c][2],
                    kf[c][3]);
#pragma unroll
        for (int c = 0; c < KQ; c++)
            ldsm_x4_t(Vs + ((size_t)(row0 + r8) * hd + (((4 * c + m4) ^ r8) << 3)) * 2, vf[c][0], vf[c][1], vf[c][2],
                      vf[c][3]);
        // S = Q K^T for the warp's 8 tokens (two independent accumulators)
        float S0[4] = {0.f, 0.f, 0.f, 0.f}, S1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < KQ; c++) {
            mma_16816(S0, qa[2 * c][0], qa[2 * c][1], qa[2 * c][2], qa[2 * c][3], kf[c][0], kf[c][1]);
            mma_16816(S1, qa[2 * c + 1][0], qa[2 * c + 1][1], qa[2 * c + 1][2], qa[2 * c + 1][3], kf[c][2], kf[c][3]);
        }
        // V rows past the context hold stale or never-written values: a lane's
        // V fragment pairs are tokens 2tq, 2tq + 1 (probability 0 must not meet
        // a NaN).  The mask is applied in program order before the release and
        // reads every V register (the products above read every K register),
        // so the stage's shared reads are complete when it is released.
        const int n = md.n;
        const bool v0 = row0 + 2 * tq < n, v1 = row0 + 2 * tq + 1 < n;
        const uint32_t vmask = (v0 ? 0x0000ffffu : 0u) | (v1 ? 0xffff0000u : 0u);
#pragma unroll
        for (int c = 0; c < KQ; c++)
#pragma unroll
            for (int j = 0; j < 4; j++) asm volatile("and.b32 %0, %0, %1;" : "+r"(vf[c][j]) : "r"(vmask));
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);         // the stage is free; its description is in md
        // ---- online softmax: row gq (S[0], S[1]), row gq + 8 (S[2], S[3]) -------------
        const float s0 = v0 ? S0[0] + S1[0] : -INFINITY, s1 = v1 ? S0[1] + S1[1] : -INFINITY;
        const float s2 = v0 ? S0[2] + S1[2] : -INFINITY, s3 = v1 ? S0[3] + S1[3] : -INFINITY;
        float mx0 = fmaxf(s0, s1), mx1 = fmaxf(s2, s3);
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const bool up0 = mx0 > m_run[0] + PERS_SLACK, up1 = mx1 > m_run[1] + PERS_SLACK;
        if (__any_sync(0xffffffffu, up0 || up1)) {
            const float al0 = !up0 ? 1.f : m_run[0] == -INFINITY ? 0.f : exp2f(m_run[0] - mx0);
            const float al1 = !up1 ? 1.f : m_run[1] == -INFINITY ? 0.f : exp2f(m_run[1] - mx1);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                acc[b][0] *= al0; acc[b][1] *= al0;
                acc[b][2] *= al1; acc[b][3] *= al1;
            }
            l_run[0] *= al0;
            l_run[1] *= al1;
            if (up0) m_run[0] = mx0;
            if (up1) m_run[1] = mx1;
        }
        const float p0 = s0 == -INFINITY ? 0.f : exp2f(s0 - m_run[0]);
        const float p1 = s1 == -INFINITY ? 0.f : exp2f(s1 - m_run[0]);
        const float p2 = s2 == -INFINITY ? 0.f : exp2f(s2 - m_run[1]);
        const float p3 = s3 == -INFINITY ? 0.f : exp2f(s3 - m_run[1]);
        l_run[0] += p0 + p1;
        l_run[1] += p2 + p3;
        const uint32_t pa0 = h2_bits(p0, p1), pa1 = h2_bits(p2, p3);
        // ---- O += P V -------------------------------------------------------------------
#pragma unroll
        for (int c = 0; c < KQ; c++) {
            mma_1688(acc[4 * c + 0], pa0, pa1, vf[c][0]);
            mma_1688(acc[4 * c + 1], pa0, pa1, vf[c][1]);
            mma_1688(acc[4 * c + 2], pa0, pa1, vf[c][2]);
            mma_1688(acc[4 * c + 3], pa0, pa1, vf[c][3]);
        }
        if (!(md.flags & PM_LAST)) continue;

        // ---- end of an item: combine the warps (comb_full counts the warps whose
        // states are in red, comb_empty those done reading it) ------------------------------
        const int col = md.col, hk = md.hk, chunk = md.chunk;
        float lsum = l_run[0];                          // the row's weight sum: its four lanes' shares
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
        if (items > 0 && !mbar_wait(comb_empty, (uint32_t)((items - 1) & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        if (gq < G) {
            float *rw = red + ((size_t)warp * G + gq) * (hd + 2);
#pragma unroll
            for (int b = 0; b < NB; b++) {
                rw[8 * b + 2 * tq] = acc[b][0];
                rw[8 * b + 2 * tq + 1] = acc[b][1];
            }
            if (tq == 0) {
                rw[hd] = m_run[0];
                rw[hd + 1] = lsum;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(comb_full);
        if (!mbar_wait(comb_full, (uint32_t)(items & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        const int n_active = md.pos / CH + 1;           // chunks of this column
        const int q = parts % PERS_MQ;
        if (n_active > 1 && parts >= PERS_MQ &&
            !mbar_wait(&mq_empty[q], (uint32_t)(((parts / PERS_MQ) - 1) & 1), a.fault, FAULT_ATTN_WAIT)) {
            *vfail = 1;
            break;
        }
        for (int i = tid; i < G * hd; i += ATTN_THREADS) {
            const int g = i / hd, d = i % hd;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < ATTN_WARPS; w++) M = fmaxf(M, red[((size_t)w * G + g) * (hd + 2) + hd]);
            float L = 0.f, A = 0.f;
#pragma unroll
            for (int w = 0; w < ATTN_WARPS; w++) {
                const float *rw = red + ((size_t)w * G + g) * (hd + 2);
                const float mw = rw[hd];
                const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
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
            // the partial goes to the merge warp (its entry is complete when
            // every consumer warp has arrived, after its share of the stores)
            if (warp == 0 && lane == 0) mq[q] = make_int4(col, hk, n_active, 0);
            __syncwarp();
            if (lane == 0) mbar_arrive(&mq_full[q]);
            parts++;
        }
    }
    if (ended) {
        // tell the merge warp that no entry follows
        const int q = parts % PERS_MQ;
        bool ok = parts < PERS_MQ ||
                  mbar_wait(&mq_empty[q], (uint32_t)(((parts / PERS_MQ) - 1) & 1), a.fault, FAULT_ATTN_WAIT);
        if (ok) {
            if (warp == 0 && lane == 0) mq[q] = make_int4(0, 0, 0, 1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&mq_full[q]);
        } else {
            *vfail = 1;
        }
    }
    // each consumer warp counts its exit; the last one of the grid resets the
    // layer's work counters (every item warp has taken its last item by then)
    if (lane == 0 && atomicAdd(&work[1], 1) == (int)gridDim.x * ATTN_WARPS - 1) {
        work[0] = 0;
        work[1] = 0;
    }
}
