// attention.cu — split-context GQA decode attention (see attention.cuh).
#include "attention.cuh"
#include "gemv_launch.cuh"

#define ATTN_WARPS 4
#define ATTN_MAX_G 8

// E = d_head / 32 floats per lane.
template <int E>
__global__ void __launch_bounds__(ATTN_WARPS * 32) k_attn(AttnArgs a) {
    const int s = blockIdx.x, hk = blockIdx.y, col = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = 32 * E;
    const int G = a.n_heads / a.n_kv;

    pdl_wait();
    pdl_launch_dependents();

    const int pos = a.pos[col];
    if (pos < 0) return;
    const int S = a.split_tokens;
    const int t0 = s * S;
    if (t0 > pos) return;
    const int t1 = min(t0 + S, pos + 1);
    const int n_active = (pos + S) / S;
    const int srow = a.slot ? a.slot[col] : col;
    const int *pt = a.page_table + (long long)srow * a.max_pages;
    const int P = a.page_tokens;

    // queries of the G heads of this kv head, lane-sliced
    float q[ATTN_MAX_G][E];
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; g++) {
        if (g < G) {
            const float *qp = a.q + (long long)col * a.q_ld + (long long)(hk * G + g) * hd + lane * E;
#pragma unroll
            for (int e = 0; e < E; e++) q[g][e] = qp[e];
        }
    }
    float m[ATTN_MAX_G], l[ATTN_MAX_G], acc[ATTN_MAX_G][E];
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; g++) {
        m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; e++) acc[g][e] = 0.f;
    }
    const long long kv_head_off = ((long long)a.layer * 2 * a.n_kv + hk) * P * hd;   // K plane
    const long long v_plane = (long long)a.n_kv * P * hd;                            // V follows K

    for (int t = t0 + warp; t < t1; t += ATTN_WARPS) {
        const int pg = pt[t / P];
        if (pg < 0 || pg >= a.n_pages) {             // never read outside the pool
            if (lane == 0 && a.fault) atomicExch(a.fault, 4u);
            continue;
        }
        const float *kp = a.kv_pages + (long long)pg * a.page_floats + kv_head_off +
                          (long long)(t % P) * hd + lane * E;
        const float *vp = kp + v_plane;
        float k[E], v[E];
#pragma unroll
        for (int e = 0; e < E; e++) { k[e] = __ldcg(kp + e); v[e] = __ldcg(vp + e); }
#pragma unroll
        for (int g = 0; g < ATTN_MAX_G; g++) {
            if (g < G) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) d = __fmaf_rn(q[g][e], k[e], d);
                float sc = warp_sum(d) * a.scale;
                float mn = fmaxf(m[g], sc);
                float corr = expf(m[g] - mn);
                float p = expf(sc - mn);
                l[g] = __fmaf_rn(l[g], corr, p);
#pragma unroll
                for (int e = 0; e < E; e++) acc[g][e] = __fmaf_rn(acc[g][e], corr, p * v[e]);
                m[g] = mn;
            }
        }
    }

    // merge the warps of this CTA
    __shared__ float wm[ATTN_WARPS][ATTN_MAX_G], wl[ATTN_WARPS][ATTN_MAX_G];
    __shared__ float wacc[ATTN_WARPS][ATTN_MAX_G][32 * E];
    __shared__ int s_last;
#pragma unroll
    for (int g = 0; g < ATTN_MAX_G; g++) {
        if (g < G) {
            if (lane == 0) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
            for (int e = 0; e < E; e++) wacc[warp][g][lane * E + e] = acc[g][e];
        }
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += ATTN_WARPS * 32) {
        int g = i / hd, d = i % hd;
        float M = -INFINITY;
        for (int w = 0; w < ATTN_WARPS; w++) M = fmaxf(M, wm[w][g]);
        float L = 0.f, A = 0.f;
        for (int w = 0; w < ATTN_WARPS; w++) {
            float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
            L = __fmaf_rn(wl[w][g], f, L);
            A = __fmaf_rn(wacc[w][g][d], f, A);
        }
        float *pp = a.part + (((long long)col * a.n_heads + hk * G + g) * a.n_splits + s) * (hd + 2);
        pp[d] = A;
        if (d == 0) { pp[hd] = M; pp[hd + 1] = L; }
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
    for (int i = tid; i < G * hd; i += ATTN_WARPS * 32) {
        int g = i / hd, d = i % hd;
        const float *base = a.part + ((long long)col * a.n_heads + hk * G + g) * a.n_splits * (hd + 2);
        float M = -INFINITY;
        for (int sp = 0; sp < n_active; sp++) M = fmaxf(M, __ldcg(base + sp * (hd + 2) + hd));
        float L = 0.f, A = 0.f;
        for (int sp = 0; sp < n_active; sp++) {
            const float *pp = base + sp * (hd + 2);
            float f = expf(__ldcg(pp + hd) - M);
            L = __fmaf_rn(__ldcg(pp + hd + 1), f, L);
            A = __fmaf_rn(__ldcg(pp + d), f, A);
        }
        a.out[(long long)col * a.out_ld + (long long)(hk * G + g) * hd + d] = A / L;
    }
    if (tid == 0) a.counters[col * a.n_kv + hk] = 0;
}

cudaError_t attention_launch(const AttnArgs &a, int ncol, cudaStream_t st, bool pdl) {
    if (a.n_heads % a.n_kv != 0 || a.n_heads / a.n_kv > ATTN_MAX_G) return cudaErrorInvalidValue;
    if (a.split_tokens % a.page_tokens != 0 || a.n_splits < 1) return cudaErrorInvalidValue;
    dim3 grid(a.n_splits, a.n_kv, ncol);
    switch (a.d_head) {
    case 64:  return launch_k(k_attn<2>, grid, dim3(ATTN_WARPS * 32), 0, st, pdl, a);
    case 128: return launch_k(k_attn<4>, grid, dim3(ATTN_WARPS * 32), 0, st, pdl, a);
    case 32:  return launch_k(k_attn<1>, grid, dim3(ATTN_WARPS * 32), 0, st, pdl, a);
    case 256: return launch_k(k_attn<8>, grid, dim3(ATTN_WARPS * 32), 0, st, pdl, a);
    default: return cudaErrorInvalidValue;
    }
}
