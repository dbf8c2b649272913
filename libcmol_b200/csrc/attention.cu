// attention.cu — split-context GQA decode attention (see attention.cuh).
//
// One CTA = (context split s, kv head hk, column).  Its split covers
// split_tokens tokens = split_tokens / page_tokens KV pages.  Thread 0 moves the K and
// V blocks of those pages (each a contiguous page_tokens x d_head block in
// the page layout) into shared memory with cp.async.bulk on one mbarrier,
// while the warps load the queries.  Scores are then computed for all
// tokens of the split at once (warp per token, lanes over d_head), the
// softmax of the split runs per head in shared memory, and P.V is one
// thread per (head, dim) over the split.  The partial (max, sum, acc) is
// merged across splits by the last CTA to finish (atomic counter), in split
// order, so the result does not depend on scheduling.
#include "attention.cuh"
#include "gemv_launch.cuh"
#include "sync.cuh"

#define ATTN_WARPS 8
#define ATTN_THREADS (ATTN_WARPS * 32)
#define ATTN_MAX_G 8

size_t attention_smem_bytes(int d_head, int G, int split_tokens) {
    // K + V tiles, queries, scores, P.V partial sums, mbarrier
    return (size_t)2 * split_tokens * d_head * 4 + (size_t)G * d_head * 4 + (size_t)G * split_tokens * 4 +
           (size_t)ATTN_THREADS * 16 + 16;
}

// E = d_head / 32.  HD4 = d_head / 4 float4 per row.
template <int E>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn(AttnArgs a) {
    const int s = blockIdx.x, hk = blockIdx.y, col = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int hd = 32 * E, HD4 = hd / 4;
    const int G = a.n_heads / a.n_kv;
    const int S = a.split_tokens;
    const int P = a.page_tokens;

    float *Ks = reinterpret_cast<float *>(cmolcu_smem);       // [S][hd]
    float *Vs = Ks + (size_t)S * hd;                          // [S][hd]
    float *Qs = Vs + (size_t)S * hd;                          // [G][hd]
    float *Sc = Qs + (size_t)G * hd;                          // [G][S]
    float4 *Red = reinterpret_cast<float4 *>(Sc + (size_t)G * S);   // [ATTN_THREADS]
    uint64_t *bar = reinterpret_cast<uint64_t *>(Red + ATTN_THREADS);
    __shared__ float wsum[ATTN_MAX_G], wmax[ATTN_MAX_G];
    __shared__ int s_last, s_ok;

    pdl_wait();
    pdl_launch_dependents();

    const int pos = a.pos[col];
    if (pos < 0) return;
    const int t0 = s * S;
    if (t0 > pos) return;
    const int n = min(S, pos + 1 - t0);                       // tokens in this split
    const int n_active = (pos + S) / S;
    const int srow = a.slot ? a.slot[col] : col;
    const int *pt = a.page_table + (long long)srow * a.max_pages;
    const long long head_off = ((long long)a.layer * 2 * a.n_kv + hk) * P * hd;   // K block in a page
    const long long v_off = (long long)a.n_kv * P * hd;                            // V block follows

    if (tid == 0) {
        s_ok = 1;
        const int npg = (n + P - 1) / P;
        for (int i = 0; i < npg; i++) {
            int pg = pt[t0 / P + i];
            if (pg < 0 || pg >= a.n_pages) s_ok = 0;
        }
        if (s_ok) {
            mbar_init(bar, 1);
            fence_mbar_init();
            mbar_arrive_expect_tx(bar, (uint32_t)(2 * npg * P * hd * 4));
            for (int i = 0; i < npg; i++) {
                const float *kp = a.kv_pages + (long long)pt[t0 / P + i] * a.page_floats + head_off;
                bulk_g2s(Ks + (size_t)i * P * hd, kp, (uint32_t)(P * hd * 4), bar);
                bulk_g2s(Vs + (size_t)i * P * hd, kp + v_off, (uint32_t)(P * hd * 4), bar);
            }
        } else if (a.fault) {
            atomicExch(a.fault, FAULT_BAD_PAGE);
        }
    }
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
        Qs[i] = a.q[(long long)col * a.q_ld + (long long)hk * G * hd + i];
    __syncthreads();
    if (!s_ok) return;
    if (!mbar_wait(bar, 0, a.fault, FAULT_ATTN_WAIT)) return;

    // scores: one thread per (token, head).  Lane l starts its walk over the
    // row at float4 l % HD4, so the 8 lanes of a shared-memory phase touch 8
    // different 16-byte bank groups of their (different) K rows.
    {
        const float4 *K4 = reinterpret_cast<const float4 *>(Ks);
        const float4 *Q4 = reinterpret_cast<const float4 *>(Qs);
        for (int w = tid; w < n * G; w += ATTN_THREADS) {
            const int t = w % n, g = w / n;
            const float4 *kr = K4 + (size_t)t * HD4;
            const float4 *qr = Q4 + (size_t)g * HD4;
            float d0 = 0.f, d1 = 0.f;
#pragma unroll
            for (int j = 0; j < HD4; j++) {
                const int c = (j + lane) & (HD4 - 1);
                const float4 k = kr[c], q = qr[c];
                d0 = __fmaf_rn(q.x, k.x, d0);
                d1 = __fmaf_rn(q.y, k.y, d1);
                d0 = __fmaf_rn(q.z, k.z, d0);
                d1 = __fmaf_rn(q.w, k.w, d1);
            }
            Sc[g * S + t] = (d0 + d1) * a.scale;
        }
    }
    __syncthreads();
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
        if (lane == 0) { wmax[g] = m; wsum[g] = sum; }
    }
    __syncthreads();
    // P.V: item = (head, float4 of d_head); the split's tokens are divided
    // among `parts` thread groups whose float4 sums meet in shared memory.
    {
        const int items = G * HD4;
        const int parts = max(1, min(ATTN_THREADS / items, n));
        const int item = tid % items, part = tid / items;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (part < parts) {
            const int g = item / HD4, c = item % HD4;
            const float *p = Sc + g * S;
            const float4 *V4 = reinterpret_cast<const float4 *>(Vs) + c;
            const int tb = (int)((long long)n * part / parts), te = (int)((long long)n * (part + 1) / parts);
            for (int t = tb; t < te; t++) {
                const float pt_ = p[t];
                const float4 v = V4[(size_t)t * HD4];
                acc.x = __fmaf_rn(pt_, v.x, acc.x);
                acc.y = __fmaf_rn(pt_, v.y, acc.y);
                acc.z = __fmaf_rn(pt_, v.z, acc.z);
                acc.w = __fmaf_rn(pt_, v.w, acc.w);
            }
            Red[tid] = acc;
        }
        __syncthreads();
        for (int i = tid; i < items; i += ATTN_THREADS) {
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
            if (c == 0) { pp[hd] = wmax[g]; pp[hd + 1] = wsum[g]; }
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int old = atomicAdd(&a.counters[col * a.n_kv + hk], 1);
        s_last = (old == n_active - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // last CTA: merge the splits in order
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
}

template <int E>
static cudaError_t launch_e(const AttnArgs &a, dim3 grid, size_t smem, cudaStream_t st, bool pdl) {
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {   // per process: the B200s of one box share the limit
        cudaError_t e = cudaFuncSetAttribute(k_attn<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, CMOLCU_ATTN_SMEM_MAX);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    return launch_k(k_attn<E>, grid, dim3(ATTN_THREADS), smem, st, pdl, a);
}

cudaError_t attention_launch(const AttnArgs &a, int ncol, cudaStream_t st, bool pdl) {
    const int G = a.n_heads / a.n_kv;
    if (a.n_heads % a.n_kv != 0 || G > ATTN_MAX_G) return cudaErrorInvalidValue;
    if (a.split_tokens % a.page_tokens != 0 || a.n_splits < 1) return cudaErrorInvalidValue;
    const size_t smem = attention_smem_bytes(a.d_head, G, a.split_tokens);
    if (smem > CMOLCU_ATTN_SMEM_MAX) return cudaErrorInvalidValue;
    dim3 grid(a.n_splits, a.n_kv, ncol);
    switch (a.d_head) {
    case 64:  return launch_e<2>(a, grid, smem, st, pdl);
    case 128: return launch_e<4>(a, grid, smem, st, pdl);
    case 32:  return launch_e<1>(a, grid, smem, st, pdl);
    case 256: return launch_e<8>(a, grid, smem, st, pdl);
    default: return cudaErrorInvalidValue;
    }
}
