// step_kernels.cu — step begin (page tables + embedding) and the sampler.
#include "step_kernels.cuh"
#include "gemv_launch.cuh"

// ---------------------------------------------------------------------------
// Embedding row dequantisation: one value of row `row`, element i.  Every
// formula is that of src/quant.c:152-232 of the reference, evaluated with
// explicitly rounded operations so the result is bit-identical to it.
// ---------------------------------------------------------------------------
__device__ float deq_elem(const QWeight &W, long long row, int i0) {
    const int j = i0 / W.kc, i = i0 - j * W.kc;          // K-chunk, index inside it
    const uint8_t *P0 = qw_row(W, 0, j, row);
    const uint8_t *P1 = W.nplanes > 1 ? qw_row(W, 1, j, row) : nullptr;
    switch (W.dtype) {
    case DT_F32: return reinterpret_cast<const float *>(P0)[i];
    case DT_F16: return h2f(reinterpret_cast<const uint16_t *>(P0)[i]);
    case DT_Q8_0: {
        float d = h2f(reinterpret_cast<const uint16_t *>(P1)[i / 32]);
        return __fmul_rn(d, (float)(int8_t)P0[i]);
    }
    case DT_Q4_0:
    case DT_Q5_0: {
        int b = i / 32, t = i % 32;
        float d = h2f(reinterpret_cast<const uint16_t *>(P1)[b]);
        uint8_t byte = P0[b * 16 + (t & 15)];
        int q = t < 16 ? (byte & 15) : (byte >> 4);
        if (W.dtype == DT_Q4_0) return __fmul_rn(d, (float)(q - 8));
        uint32_t qh = reinterpret_cast<const uint32_t *>(qw_row(W, 2, j, row))[b];
        q |= (int)((qh >> t) & 1u) << 4;
        return __fmul_rn(d, (float)(q - 16));
    }
    case DT_Q4_K: {
        int sb = i / 256, w = i % 256, sub = w / 32, l = w % 32;
        const uint8_t *h = P1 + sb * 16;
        float d = h2f((uint16_t)(h[0] | (h[1] << 8)));
        float dmin = h2f((uint16_t)(h[2] | (h[3] << 8)));
        const uint8_t *s = h + 4;
        int sc, mn;
        if (sub < 4) { sc = s[sub] & 63; mn = s[sub + 4] & 63; }
        else { sc = (s[sub + 4] & 15) | ((s[sub - 4] >> 6) << 4); mn = (s[sub + 4] >> 4) | ((s[sub] >> 6) << 4); }
        uint8_t byte = P0[sb * 128 + (sub / 2) * 32 + l];
        int nib = (sub & 1) ? (byte >> 4) : (byte & 15);
        float db = __fmul_rn(d, (float)sc), mb = __fmul_rn(dmin, (float)mn);
        return __fsub_rn(__fmul_rn(db, (float)nib), mb);
    }
    case DT_Q6_K: {
        int sb = i / 256, w = i % 256, g = w / 32, t = w % 32;
        int lo = (P0[sb * 128 + (g < 4 ? 0 : 64) + (g & 1) * 32 + t] >> ((g & 2) ? 4 : 0)) & 15;
        int hi = (P1[sb * 64 + (g < 4 ? 0 : 32) + t] >> ((g & 3) * 2)) & 3;
        int q = (lo | (hi << 4)) - 32;
        float sc = (float)(int8_t)qw_row(W, 2, j, row)[sb * 16 + w / 16];
        float d = h2f(reinterpret_cast<const uint16_t *>(qw_row(W, 3, j, row))[sb]);
        return __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
    default: return 0.f;
    }
}

__global__ void k_step_begin(StepBeginArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    const int col = blockIdx.x;
    if (col == 0 && threadIdx.x == 0 && *a.meta.stall) {
        // fault-path test: a wait on a barrier that nothing arrives on, bounded
        // by polling (mbarrier.test_wait never suspends: ~2^20 polls, a few ms),
        // records its code like every other wait that runs out
        __shared__ uint64_t never;
        mbar_init(&never, 1);
        fence_mbar_init();
        bool done = false;
        for (uint32_t i = 0; i < (1u << 20) && !done; i++) {
            uint32_t ok;
            asm volatile(
                "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(ok)
                : "r"(smem_u32(&never))
                : "memory");
            done = ok != 0;
        }
        if (!done && a.fault) atomicExch(a.fault, FAULT_STEP_WAIT);
    }
    if (col == 0) {
        const int n = *a.meta.n_upd;
        for (int u = threadIdx.x; u < n; u += blockDim.x) {
            int s = a.meta.upd[3 * u], idx = a.meta.upd[3 * u + 1], pg = a.meta.upd[3 * u + 2];
            if (s < 0 || s >= a.max_slots || idx < 0 || idx >= a.max_pages || pg < 0 || pg >= a.n_pages) {
                if (a.fault) atomicExch(a.fault, FAULT_BAD_PAGE);
                continue;
            }
            a.page_table[(long long)s * a.max_pages + idx] = pg;
        }
    }
    if (a.meta.pos[col] < 0) return;
    const int tok = a.meta.token[col];
    float *x = a.x + (long long)col * a.d_model;
    if (tok < 0 || tok >= a.embd.rows) {        // never read outside the table
        if (threadIdx.x == 0 && a.fault) atomicExch(a.fault, FAULT_BAD_TOKEN);
        for (int i = threadIdx.x; i < a.d_model; i += blockDim.x) x[i] = 0.f;
        return;
    }
    for (int i = threadIdx.x; i < a.d_model; i += blockDim.x) x[i] = deq_elem(a.embd, tok, i);
}

cudaError_t step_begin_launch(const StepBeginArgs &a, int ncol, cudaStream_t st, bool pdl) {
    return launch_k(k_step_begin, dim3(ncol), dim3(256), 0, st, pdl, a);
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE + KV append.  Block = (column, head); heads [0, n_heads)
// are query heads, [n_heads, n_heads + n_kv) key/value heads.
// ---------------------------------------------------------------------------
__global__ void k_qknorm(QkNormArgs a, int n_heads) {
    pdl_wait();
    pdl_launch_dependents();
    const int col = blockIdx.x, h = blockIdx.y, lane = threadIdx.x;
    const EpiQKV &e = a.e;
    const int pos = e.pos[col];
    if (pos < 0) return;
    const int hd = e.d_head, D = e.d_model, KVD = e.kv_dim;
    const bool is_q = h < n_heads;
    const int kh = h - n_heads;
    const float *src = a.qkv + (long long)col * a.qkv_ld + (is_q ? h * hd : D + kh * hd);
    const float *w = is_q ? a.q_norm : a.k_norm;
    float v[8];                                  // hd <= 256
    float ss = 0.f;
    for (int i = 0; i < hd / 32; i++) { v[i] = src[lane + 32 * i]; ss = __fmaf_rn(v[i], v[i], ss); }
    if (w) {
        ss = warp_sum(ss);
        float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
        for (int i = 0; i < hd / 32; i++) v[i] = __fmul_rn(w[lane + 32 * i], __fmul_rn(v[i], inv));
    }
    // pairs (2j, 2j+1) live in adjacent lanes
    float out[8];
    for (int i = 0; i < hd / 32; i++) {
        int idx = lane + 32 * i;
        float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
        float r = v[i];
        if (e.rope) {
            float2 cs = e.rope_cs[(long long)pos * (hd / 2) + (idx >> 1)];
            r = (idx & 1) ? __fadd_rn(__fmul_rn(other, cs.y), __fmul_rn(v[i], cs.x))
                          : __fsub_rn(__fmul_rn(v[i], cs.x), __fmul_rn(other, cs.y));
        }
        out[i] = r;
    }
    if (is_q) {
        float *q = a.q_out + (long long)col * a.q_ld + h * hd;
        for (int i = 0; i < hd / 32; i++) q[lane + 32 * i] = out[i];
        return;
    }
    const int srow = e.slot ? e.slot[col] : col;
    const int pg = e.page_table[(long long)srow * e.max_pages + pos / e.page_tokens];
    if (pg < 0 || pg >= e.n_pages) return;
    const int t = pos % e.page_tokens;
    const long long ko = (long long)pg * e.page_elems + ((long long)kh * 2 * e.page_tokens + t) * hd;
    const long long vo = ko + (long long)e.page_tokens * hd;     // the head's V block follows its K block
    const float *vsrc = a.qkv + (long long)col * a.qkv_ld + D + KVD + kh * hd;
    for (int i = 0; i < hd / 32; i++) {
        const int j = lane + 32 * i;
        if (e.kv_f16) {
            const int js = kv_swz(pos, j, hd);
            static_cast<__half *>(e.kv_pages)[ko + js] = __float2half_rn(out[i]);
            static_cast<__half *>(e.kv_pages)[vo + js] = __float2half_rn(vsrc[j]);
        } else {
            static_cast<float *>(e.kv_pages)[ko + j] = out[i];
            static_cast<float *>(e.kv_pages)[vo + j] = vsrc[j];
        }
    }
}

cudaError_t qknorm_launch(const QkNormArgs &a, int ncol, int n_heads, cudaStream_t st, bool pdl) {
    if (a.e.d_head % 32 || a.e.d_head > 256) return cudaErrorInvalidValue;
    return launch_k(k_qknorm, dim3(ncol, n_heads + a.e.n_kv), dim3(32), 0, st, pdl, a, n_heads);
}

// ---------------------------------------------------------------------------
// Sampler: one CTA per column.  src/sampler.c:171-268 + the repeat ring of
// src/api.c:465-507.
// ---------------------------------------------------------------------------
#define SMP_THREADS 1024
#define SMP_WARPS (SMP_THREADS / 32)

__device__ __forceinline__ unsigned long long rotl64(unsigned long long x, int k) {
    return (x << k) | (x >> (64 - k));
}

// xoshiro256** step (src/sampler.c:37-49)
__device__ unsigned long long rng_next(unsigned long long *s) {
    unsigned long long r = rotl64(s[1] * 5ull, 7) * 9ull;
    unsigned long long t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return r;
}

// uniform [0,1) from the top 23 bits (src/sampler.c:78-84)
__device__ float rng_unit(unsigned long long *s) {
    unsigned int bits = 0x3F800000u | (unsigned int)(rng_next(s) >> 41);
    return __uint_as_float(bits) - 1.0f;
}

__device__ float block_max(float v, float *red) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < SMP_WARPS ? red[lane] : -INFINITY;
        t = warp_max(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

__device__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < SMP_WARPS ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// argmax with ties to the lowest index (src/sampler.c:199-204)
__device__ int block_argmax(const float *x, int n, float *redv, int *redi) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += SMP_THREADS) {
        float v = x[i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { redv[warp] = bv; redi[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        bv = lane < SMP_WARPS ? redv[lane] : -INFINITY;
        bi = lane < SMP_WARPS ? redi[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) redi[0] = bi;
    }
    __syncthreads();
    int r = redi[0];
    return r == 0x7fffffff ? 0 : r;
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(SampleArgs a) {
    __shared__ float redv[SMP_WARPS];
    __shared__ int redi[SMP_WARPS];
    __shared__ unsigned int hist[256];
    __shared__ int s_sel, s_krem, s_ngt;
    __shared__ float cval[CMOLCU_TOPK_MAX];
    __shared__ int cidx[CMOLCU_TOPK_MAX];
    __shared__ int eq_scan[SMP_THREADS];

    pdl_wait();
    pdl_launch_dependents();

    const int col = blockIdx.x, tid = threadIdx.x;
    if (a.meta.pos[col] < 0 || !a.meta.sample[col]) return;
    const int V = a.vocab;
    float *L = a.logits + (long long)col * V;
    SlotSampler *st = a.slots + a.meta.slot[col];

    // repeat penalty, applied in ring order (src/sampler.c:171-184)
    if (tid == 0 && st->repeat_penalty > 1.0f && st->ring_fill > 0) {
        for (int i = 0; i < st->ring_fill; i++) {
            int id = st->ring[i];
            if (id < 0 || id >= V) continue;
            if (L[id] > 0.0f) L[id] = __fdiv_rn(L[id], st->repeat_penalty);
            else L[id] = __fmul_rn(L[id], st->repeat_penalty);
        }
    }
    __syncthreads();

    int token;
    if (st->temperature == 0.0f) {
        token = block_argmax(L, V, redv, redi);
    } else {
        // temperature, softmax (src/sampler.c:207-213)
        const float inv_t = __fdiv_rn(1.0f, st->temperature);
        float mx = -INFINITY;
        for (int i = tid; i < V; i += SMP_THREADS) {
            float v = __fmul_rn(L[i], inv_t);
            L[i] = v;
            mx = fmaxf(mx, v);
        }
        mx = block_max(mx, redv);
        float sm = 0.f;
        for (int i = tid; i < V; i += SMP_THREADS) {
            float e = expf(__fsub_rn(L[i], mx));
            L[i] = e;
            sm += e;
        }
        sm = block_sum(sm, redv);
        const float inv = __fdiv_rn(1.0f, sm);
        for (int i = tid; i < V; i += SMP_THREADS) L[i] = __fmul_rn(L[i], inv);
        __syncthreads();

        const int use_k = st->top_k > 0 && st->top_k < V;
        const int use_p = st->top_p > 0.0f && st->top_p < 1.0f;
        if (!use_k && !use_p) {
            // categorical CDF walk over the whole vocabulary (src/sampler.c:219-234),
            // kept sequential so the float prefix sums are the reference's.
            if (tid == 0) {
                float r = rng_unit(st->rng), acc = 0.f;
                int pick = V - 1;
                for (int i = 0; i < V - 1; i++) {
                    acc = __fadd_rn(acc, L[i]);
                    if (r < acc) { pick = i; break; }
                }
                s_sel = pick;
            }
            __syncthreads();
            token = s_sel;
        } else {
            int k = use_k ? st->top_k : V;
            if (k > CMOLCU_TOPK_MAX) k = CMOLCU_TOPK_MAX;
            // radix select of the k-th largest probability (bits of p >= 0 are monotonic)
            unsigned int prefix = 0, mask = 0;
            if (tid == 0) s_krem = k;
            for (int shift = 24; shift >= 0; shift -= 8) {
                for (int b = tid; b < 256; b += SMP_THREADS) hist[b] = 0;
                __syncthreads();
                for (int i = tid; i < V; i += SMP_THREADS) {
                    unsigned int u = __float_as_uint(L[i]);
                    if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
                }
                __syncthreads();
                if (tid == 0) {
                    int krem = s_krem, cum = 0, sel = 0;
                    for (int b = 255; b >= 0; b--) {
                        if (cum + (int)hist[b] >= krem) { sel = b; krem -= cum; break; }
                        cum += hist[b];
                    }
                    s_sel = sel;
                    s_krem = krem;
                }
                __syncthreads();
                prefix |= (unsigned int)s_sel << shift;
                mask |= 255u << shift;
            }
            const int n_eq_take = s_krem;          // elements equal to the threshold to keep
            const int n_gt = k - n_eq_take;        // elements strictly above it
            if (tid == 0) s_ngt = 0;
            for (int i = tid; i < CMOLCU_TOPK_MAX; i += SMP_THREADS) { cval[i] = -1.0f; cidx[i] = -1; }
            __syncthreads();
            // strictly greater: unordered append (sorted below)
            for (int i = tid; i < V; i += SMP_THREADS) {
                unsigned int u = __float_as_uint(L[i]);
                if (u > prefix) {
                    int p = atomicAdd(&s_ngt, 1);
                    if (p < CMOLCU_TOPK_MAX) { cval[p] = L[i]; cidx[p] = i; }
                }
            }
            // equal to the threshold: the lowest indices first (block-ordered scan)
            const int chunk = (V + SMP_THREADS - 1) / SMP_THREADS;
            const int i0 = tid * chunk, i1 = min(V, i0 + chunk);
            int cnt = 0;
            for (int i = i0; i < i1; i++) cnt += (__float_as_uint(L[i]) == prefix);
            eq_scan[tid] = cnt;
            __syncthreads();
            if (tid == 0) {
                int run = 0;
                for (int t = 0; t < SMP_THREADS; t++) { int c = eq_scan[t]; eq_scan[t] = run; run += c; }
            }
            __syncthreads();
            int rank = eq_scan[tid];
            for (int i = i0; i < i1 && rank < n_eq_take; i++) {
                if (__float_as_uint(L[i]) == prefix) {
                    int p = n_gt + rank;
                    if (p < CMOLCU_TOPK_MAX) { cval[p] = L[i]; cidx[p] = i; }
                    rank++;
                }
            }
            __syncthreads();
            // bitonic sort: value descending, index ascending (512 slots)
            for (int i = tid; i < CMOLCU_TOPK_MAX; i += SMP_THREADS)
                if (i >= k) { cval[i] = -1.0f; cidx[i] = 0x7fffffff; }
            __syncthreads();
            for (int size = 2; size <= CMOLCU_TOPK_MAX; size <<= 1) {
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    if (tid < CMOLCU_TOPK_MAX) {
                        int j = tid ^ stride;
                        if (j > tid) {
                            bool desc = (tid & size) == 0;
                            float vi = cval[tid], vj = cval[j];
                            int ii = cidx[tid], ij = cidx[j];
                            bool i_first = (vi > vj) || (vi == vj && ii < ij);
                            if (desc ? !i_first : i_first) {
                                cval[tid] = vj; cval[j] = vi; cidx[tid] = ij; cidx[j] = ii;
                            }
                        }
                    }
                    __syncthreads();
                }
            }
            // nucleus, renormalise, CDF walk: sequential as src/sampler.c:245-267
            if (tid == 0) {
                int nucleus = k;
                if (use_p) {
                    float cum = 0.f;
                    for (int i = 0; i < k; i++) {
                        cum = __fadd_rn(cum, cval[i]);
                        if (cum >= st->top_p) { nucleus = i + 1; break; }
                    }
                }
                float sum = 0.f;
                for (int i = 0; i < nucleus; i++) sum = __fadd_rn(sum, cval[i]);
                int pick = cidx[0];
                if (sum > 0.0f) {
                    float r = __fmul_rn(rng_unit(st->rng), sum), acc = 0.f;
                    pick = cidx[nucleus - 1];
                    for (int i = 0; i < nucleus; i++) {
                        acc = __fadd_rn(acc, cval[i]);
                        if (r < acc) { pick = cidx[i]; break; }
                    }
                }
                s_sel = pick;
            }
            __syncthreads();
            token = s_sel;
        }
    }
    if (tid == 0) {
        if (token < 0 || token >= V) {          // non-finite logits leave no valid candidate
            if (a.fault) atomicExch(a.fault, FAULT_SAMPLE);
            token = 0;
        }
        a.out_ids[col] = token;
        if (!(st->eos >= 0 && token == st->eos)) {       // src/api.c:502-507
            st->ring[st->ring_head] = token;
            st->ring_head = (st->ring_head + 1) % CMOLCU_REPEAT_BUF;
            if (st->ring_fill < CMOLCU_REPEAT_BUF) st->ring_fill++;
        }
    }
}

cudaError_t sample_launch(const SampleArgs &a, int ncol, cudaStream_t st, bool pdl) {
    return launch_k(k_sample, dim3(ncol), dim3(SMP_THREADS), 0, st, pdl, a);
}
