// attention.cu — standalone launch of the split-context GQA decode attention
// item (attention_item.cuh): one CTA per (split, kv head, column).
#include "attention_item.cuh"
#include "gemv_launch.cuh"

size_t attention_smem_bytes(int d_head, int G, int split_tokens) {
    return attn_item_smem_bytes(d_head, G, split_tokens) + 16;   // + the mbarrier
}

// One CTA per item: grid (split, kv head, column).
template <int E>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn(AttnArgs a) {
    const int G = a.n_heads / a.n_kv;
    float *sm = reinterpret_cast<float *>(cmolcu_smem);
    uint64_t *bar = reinterpret_cast<uint64_t *>(cmolcu_smem + attn_item_smem_bytes(32 * E, G, a.split_tokens));
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
    attn_item<E>(a, blockIdx.x, blockIdx.y, col, pos, a.page_table + (long long)srow * a.max_pages, sm, bar, parity,
                 sh, threadIdx.x);
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
