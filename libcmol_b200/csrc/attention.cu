// attention.cu — standalone launch of the split-context GQA decode attention
// item (attention_item.cuh): one CTA per (split, kv head, column).
#include "attention_decode.cuh"
#include "attention_item.cuh"
#include "gemv_launch.cuh"

#include <stdlib.h>

#include <algorithm>

size_t attention_smem_bytes(int d_head, int G, int split_tokens, int q_chunk, int kvb) {
    return attn_group_smem_bytes(d_head, G, split_tokens, q_chunk, kvb) + 16;   // + the mbarrier
}

int attention_q_chunk(int d_head, int G, int split_tokens) {
    // 6 KB: configs 1-4 keep the CTAs per SM of the one-query layout, but for
    // SmolLM2-1.7B's (G = 1), which goes from 6 to 5
    return attn_group_qc(d_head, G, split_tokens, 6 * 1024);
}


// Steps without prefill groups: one CTA per (split, kv head, column), each
// running attn_item.
template <int E, bool H>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn(AttnArgs a) {
    const int G = a.n_heads / a.n_kv;
    float *sm = reinterpret_cast<float *>(cmolcu_smem);
    uint64_t *bar =
        reinterpret_cast<uint64_t *>(cmolcu_smem + attn_item_smem_bytes(32 * E, G, a.split_tokens, H ? 2 : 4));
    __shared__ AttnShared sh;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    pdl_wait();
    pdl_launch_dependents();
    named_bar_sync(1, ATTN_THREADS);
    uint32_t parity = 0;
    const int col = blockIdx.z;
    const int pos = a.pos[col];
    const int srow = a.slot ? a.slot[col] : col;
    attn_item<E, H>(a, blockIdx.x, blockIdx.y, col, pos, a.page_table + (long long)srow * a.max_pages, sm, bar,
                    parity, sh, threadIdx.x);
}

// Steps with prefill groups: one CTA per (split, kv head, column).  A column
// alone in its session (decode) runs attn_item; the columns of a prefill
// group are served by their block leaders (attn_group_item).  CTAs per SM
// that the shared memory of the engine's shapes allows (d_head 64: 5, 128:
// 3); registers are held to that.
template <int E, bool H>
__global__ void __launch_bounds__(ATTN_THREADS, E <= 2 ? 5 : E == 4 ? 3 : 2) k_attn_group(AttnArgs a) {
    const int G = a.n_heads / a.n_kv;
    float *sm = reinterpret_cast<float *>(cmolcu_smem);
    uint64_t *bar = reinterpret_cast<uint64_t *>(
        cmolcu_smem + attn_group_smem_bytes(32 * E, G, a.split_tokens, a.q_chunk, H ? 2 : 4));
    __shared__ union {
        AttnShared      one;
        AttnGroupShared grp;
    } sh;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    pdl_wait();
    pdl_launch_dependents();
    named_bar_sync(1, ATTN_THREADS);
    uint32_t parity = 0;
    const int c = blockIdx.z, ncol = gridDim.z;
    // the column and its neighbours, loaded together
    const int cp = c > 0 ? c - 1 : c, cn = c + 1 < ncol ? c + 1 : c;
    const int pos = a.pos[c], pos_p = a.pos[cp], pos_n = a.pos[cn];
    int slot = c, slot_p = cp, slot_n = cn;
    if (a.slot) { slot = a.slot[c]; slot_p = a.slot[cp]; slot_n = a.slot[cn]; }
    const bool grouped = a.slot && a.grouped;
    const bool prev = grouped && cp != c && slot_p == slot && pos_p == pos - 1;
    const bool next = grouped && cn != c && slot_n == slot && pos_n == pos + 1;
    if (pos >= 0 && (prev || next))
        attn_group_item<E, H>(a, blockIdx.x, blockIdx.y, c, pos, slot, next, sm, bar, parity, sh.grp, threadIdx.x);
    else
        attn_item<E, H>(a, blockIdx.x, blockIdx.y, c, pos, a.page_table + (long long)slot * a.max_pages, sm, bar,
                        parity, sh.one, threadIdx.x);
}

// Work-list launch (opt-in): a fixed grid of a few CTAs per SM; each
// CTA lists the active (column, kv head, split) items of the step from the
// columns' positions (prefix sum over columns in shared memory) and takes
// items blockIdx.x, blockIdx.x + gridDim.x, ...  The grid then depends on the
// SM count, not on the longest context the pool allows, so steps whose
// sessions are short do not pay for launching (and retiring) the splits they
// do not have.
#define ATTN_LIST_MAX_COLS 1024

template <int E, bool H>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn_list(AttnArgs a, int ncol) {
    const int G = a.n_heads / a.n_kv;
    float *sm = reinterpret_cast<float *>(cmolcu_smem);
    uint64_t *bar =
        reinterpret_cast<uint64_t *>(cmolcu_smem + attn_item_smem_bytes(32 * E, G, a.split_tokens, H ? 2 : 4));
    __shared__ AttnShared sh;
    __shared__ int start[ATTN_LIST_MAX_COLS + 1];   // start[c] = first item of column c
    __shared__ int wsum[ATTN_WARPS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    pdl_wait();
    pdl_launch_dependents();
    // items per column, then an exclusive prefix sum (chunks of ATTN_THREADS columns)
    const int S = a.split_tokens;
    int carry = 0;
    for (int c0 = 0; c0 < ncol; c0 += ATTN_THREADS) {
        const int c = c0 + tid;
        int n = 0;
        if (c < ncol) {
            const int pos = a.pos[c];
            n = pos < 0 ? 0 : a.n_kv * (pos / S + 1);
        }
        int v = n;   // inclusive scan within the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        if (lane == 31) wsum[warp] = v;
        named_bar_sync(1, ATTN_THREADS);
        int before = carry;
        for (int w = 0; w < warp; w++) before += wsum[w];
        if (c < ncol) start[c] = before + v - n;
        int tot = 0;
        for (int w = 0; w < ATTN_WARPS; w++) tot += wsum[w];
        carry += tot;
        named_bar_sync(1, ATTN_THREADS);
    }
    if (tid == 0) start[ncol] = carry;
    named_bar_sync(1, ATTN_THREADS);
    const int total = carry;
    uint32_t parity = 0;
    for (int i = blockIdx.x; i < total; i += gridDim.x) {
        int lo = 0, hi = ncol - 1;          // last column with start <= i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (start[mid] <= i) lo = mid; else hi = mid - 1;
        }
        const int col = lo, r = i - start[col];
        const int nsp = (start[col + 1] - start[col]) / a.n_kv;
        const int hk = r / nsp, sp = r % nsp;
        const int pos = a.pos[col];
        const int srow = a.slot ? a.slot[col] : col;
        if (!attn_item<E, H>(a, sp, hk, col, pos, a.page_table + (long long)srow * a.max_pages, sm, bar, parity, sh,
                             tid))
            return;   // fault recorded (uniform over the CTA)
    }
}

template <int E, bool H>
static cudaError_t launch_e(const AttnArgs &a, int ncol, size_t smem, cudaStream_t st, bool pdl) {
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {   // per process: the B200s of one box share the limit
        cudaError_t e =
            cudaFuncSetAttribute(k_attn<E, H>, cudaFuncAttributeMaxDynamicSharedMemorySize, CMOLCU_ATTN_SMEM_MAX);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_group<E, H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     CMOLCU_ATTN_SMEM_MAX);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_list<E, H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     CMOLCU_ATTN_SMEM_MAX);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    const int sms = device_sm_count();
    const int per_sm = std::max(1, std::min(4, (int)((200 * 1024) / (smem + 8 * 1024))));
    // The grid launch (one CTA per item, inactive splits exit at once) measured
    // faster at every size tried: 5.31 against 6.94 ms/step on config 3 (~51 K
    // cells) and 15.8 against 50.3 ms/step on config 4 (~136 K cells), since it
    // keeps far more items in flight than a few CTAs per SM walking a list.
    // CMOLCU_ATTN_LIST=1 selects the work-list launch (tests, measurements).
    static const bool force_list = [] {
        const char *v = getenv("CMOLCU_ATTN_LIST");
        return v && v[0] == '1';
    }();
    const bool list = force_list;
    if (list && ncol <= ATTN_LIST_MAX_COLS)   // per-column items (no prefill groups)
        return launch_k(k_attn_list<E, H>, dim3(sms * per_sm), dim3(ATTN_THREADS), smem, st, pdl, a, ncol);
    if (a.grouped)
        return launch_k(k_attn_group<E, H>, dim3(a.n_splits, a.n_kv, ncol), dim3(ATTN_THREADS), smem, st, pdl, a);
    return launch_k(k_attn<E, H>, dim3(a.n_splits, a.n_kv, ncol), dim3(ATTN_THREADS), smem, st, pdl, a);
}

// Ring stages of the decode kernel: about 96 KB of K / V in flight per CTA
// (two CTAs an SM), at least two stages.
static int dec_stages(int hd, int kvb) {
    const size_t stage = (size_t)2 * DEC_SUB * hd * kvb;
    int s = (int)((96 * 1024) / stage);
    return s < 2 ? 2 : s > 4 ? 4 : s;
}

template <int E, bool H, int GP>
static cudaError_t launch_dec(const AttnArgs &a, int ncol, cudaStream_t st, bool pdl) {
    const int kvb = H ? 2 : 4, stages = dec_stages(32 * E, kvb);
    const size_t smem = dec_smem_bytes(32 * E, kvb, GP, stages);
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_dec<E, H, GP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
    }
    const int n_chunks = (a.n_splits * a.split_tokens + a.chunk_tokens - 1) / a.chunk_tokens;
    return launch_k(k_attn_dec<E, H, GP>, dim3(n_chunks, a.n_kv, ncol), dim3(ATTN_THREADS), smem, st, pdl, a,
                    stages);
}

#define PERS_SMEM_BUDGET (227 * 1024)

template <int E>
static cudaError_t launch_pers(const AttnArgs &a, cudaStream_t st, bool pdl) {
    const int G = a.n_heads / a.n_kv;
    const int stages = pers_stages(32 * E, G, a.max_cols, PERS_SMEM_BUDGET);
    const size_t smem = pers_fixed_bytes(32 * E, G, a.max_cols) + (size_t)stages * pers_stage_bytes(32 * E, G);
    static int attr_dev = -1;
    static size_t attr_smem = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev || attr_smem < smem) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_pers<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_dev = dev;
        attr_smem = smem;
    }
    return launch_k(k_attn_pers<E>, dim3(device_sm_count()), dim3(PERS_THREADS), smem, st, pdl, a, stages,
                    a.max_cols);
}

template <int E, bool H>
static cudaError_t launch_dec_g(const AttnArgs &a, int ncol, cudaStream_t st, bool pdl) {
    switch (dec_pow2(a.n_heads / a.n_kv)) {
    case 1: return launch_dec<E, H, 1>(a, ncol, st, pdl);
    case 2: return launch_dec<E, H, 2>(a, ncol, st, pdl);
    case 4: return launch_dec<E, H, 4>(a, ncol, st, pdl);
    default: return launch_dec<E, H, 8>(a, ncol, st, pdl);
    }
}

cudaError_t attention_launch(const AttnArgs &a_in, int ncol, cudaStream_t st, bool pdl) {
    AttnArgs a = a_in;
    const int G = a.n_heads / a.n_kv;
    if (a.n_heads % a.n_kv != 0 || G > ATTN_MAX_G) return cudaErrorInvalidValue;
    if (a.split_tokens % a.page_tokens != 0 || a.n_splits < 1) return cudaErrorInvalidValue;
    if (a.q_chunk < 1 || a.q_chunk > ATTN_QB || a.q_block < 1 || a.q_block > ATTN_QB) return cudaErrorInvalidValue;
    // the group layout (a superset of the one-query layout) bounds both kernels
    const int kvb = a.kv_f16 ? 2 : 4;
    static const bool force_list = [] {
        const char *v = getenv("CMOLCU_ATTN_LIST");
        return v && v[0] == '1';
    }();
    static const bool split_items = [] {
        const char *v = getenv("CMOLCU_ATTN_DECODE");
        return v && v[0] == '0';
    }();
    // Decode steps (one token per session): the streaming kernel of
    // attention_decode.cuh, with chunks of 64..512 tokens, longer when the
    // step has more (column, kv head) pairs to spread over the SMs.
    if (!a.grouped && !force_list && !split_items && (a.d_head == 64 || a.d_head == 128) &&
        DEC_SUB % a.page_tokens == 0 && a.split_tokens <= DEC_SUB) {
        // CMOLCU_ATTN_SUBS fixes the 64-token sub-tiles a chunk (measurement switch)
        static const int subs_knob = [] {
            const char *v = getenv("CMOLCU_ATTN_SUBS");
            return v && *v ? atoi(v) : 0;
        }();
        int subs = 1;
        while (subs < 8 && ncol * a.n_kv >= 64 * subs) subs <<= 1;
        if (subs_knob == 1 || subs_knob == 2 || subs_knob == 4 || subs_knob == 8) subs = subs_knob;
        a.chunk_tokens = DEC_SUB * subs;
        const bool h = a.kv_f16 != 0;
        if (h && a.tc_min_cols > 0 && ncol >= a.tc_min_cols && a.order && a.work &&
            pers_stages(a.d_head, G, a.max_cols, PERS_SMEM_BUDGET) >= 2)
            return a.d_head == 64 ? launch_pers<2>(a, st, pdl) : launch_pers<4>(a, st, pdl);
        if (a.d_head == 64) return h ? launch_dec_g<2, true>(a, ncol, st, pdl) : launch_dec_g<2, false>(a, ncol, st, pdl);
        return h ? launch_dec_g<4, true>(a, ncol, st, pdl) : launch_dec_g<4, false>(a, ncol, st, pdl);
    }
    if (attention_smem_bytes(a.d_head, G, a.split_tokens, a.q_chunk, kvb) > CMOLCU_ATTN_SMEM_MAX)
        return cudaErrorInvalidValue;
    const size_t smem = a.grouped ? attention_smem_bytes(a.d_head, G, a.split_tokens, a.q_chunk, kvb)
                                  : attn_item_smem_bytes(a.d_head, G, a.split_tokens, kvb) + 16;
    const bool h = a.kv_f16 != 0;
    switch (a.d_head) {
    case 64:  return h ? launch_e<2, true>(a, ncol, smem, st, pdl) : launch_e<2, false>(a, ncol, smem, st, pdl);
    case 128: return h ? launch_e<4, true>(a, ncol, smem, st, pdl) : launch_e<4, false>(a, ncol, smem, st, pdl);
    case 32:  return h ? launch_e<1, true>(a, ncol, smem, st, pdl) : launch_e<1, false>(a, ncol, smem, st, pdl);
    case 256: return h ? launch_e<8, true>(a, ncol, smem, st, pdl) : launch_e<8, false>(a, ncol, smem, st, pdl);
    default: return cudaErrorInvalidValue;
    }
}
