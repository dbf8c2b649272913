// sync.cuh — mbarrier / bulk-copy / named-barrier helpers (inline PTX,
// sm_90+ forms valid on sm_100a) and the device fault word.
//
// Every wait is bounded: after CMOLCU_SPIN_LIMIT unsuccessful try_wait
// calls the waiter records a fault code in the caller's device fault word
// (a kernel argument; NULL = do not record) and gives up, so a lost arrival
// can never hang the GPU.  The host reads the word after the step.
#pragma once
#include "common.cuh"

#define CMOLCU_SPIN_LIMIT (1u << 22)

enum : unsigned int {
    FAULT_NONE = 0,
    FAULT_GEMV_FULL = 1,       // consumer waited too long for a stage
    FAULT_GEMV_EMPTY = 2,      // producer waited too long for a free stage
    FAULT_BAD_TOKEN = 3,       // a token id outside [0, vocab) reached the embedding
    FAULT_BAD_PAGE = 4,        // a page-table update outside the table / pool
    FAULT_SAMPLE = 5,          // the sampler found no valid candidate (non-finite logits)
    FAULT_ATTN_WAIT = 6,       // attention waited too long for its K/V pages
    FAULT_STEP_WAIT = 7,       // the step-begin kernel's wait ran out (cmol_cuda_debug_inject kind 3)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned int *fault_word,
                                          unsigned int code) {
    for (uint32_t i = 0; i < CMOLCU_SPIN_LIMIT; i++)
        if (mbar_try_wait(bar, parity)) return true;
    if (fault_word) atomicExch(fault_word, code);
    return false;
}

// Global -> shared bulk copy (non-tensor TMA), completion counted in bytes on
// `bar`.  dst, src and size must be multiples of 16 bytes.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
