// common.cuh — shared helpers for the libcmol B200 engine (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#ifndef __CUDACC__
#error "compile with nvcc"
#endif

#define CMOLCU_WARP 32

// GGUF tensor type tags (same numbering as the GGUF format and as
// src/cmol_internal.h:27-37 of the reference).
enum : int {
    DT_F32 = 0, DT_F16 = 1, DT_Q4_0 = 2, DT_Q5_0 = 6, DT_Q8_0 = 8,
    DT_Q4_K = 12, DT_Q6_K = 14
};

__host__ __device__ inline int dt_block_values(int dt) {
    switch (dt) {
    case DT_F32: case DT_F16: return 1;
    case DT_Q4_0: case DT_Q5_0: case DT_Q8_0: return 32;
    case DT_Q4_K: case DT_Q6_K: return 256;
    default: return 0;
    }
}

__host__ __device__ inline int dt_block_bytes(int dt) {
    switch (dt) {
    case DT_F32: return 4;
    case DT_F16: return 2;
    case DT_Q4_0: return 18;
    case DT_Q5_0: return 22;
    case DT_Q8_0: return 34;
    case DT_Q4_K: return 144;
    case DT_Q6_K: return 210;
    default: return 0;
    }
}

__host__ __device__ inline size_t dt_row_bytes(int k, int dt) {
    int bv = dt_block_values(dt);
    return bv ? (size_t)(k / bv) * (size_t)dt_block_bytes(dt) : 0;
}

// f16 KV pages store each token's d_head values with their 16-byte chunks
// (8 values) permuted by the token's position in the context: chunk c of the
// token at position pos sits at chunk c ^ (pos & m), m = min(7, chunks per
// row - 1).  Eight consecutive positions then place any one chunk in eight
// different bank groups, so the tensor-core fragment loads (ldmatrix) of K
// and V tiles are free of bank conflicts.  Stored index of value d.
__host__ __device__ __forceinline__ int kv_swz(int pos, int d, int hd) {
    const int m = hd >= 64 ? 7 : (hd >> 3) - 1;
    return (((d >> 3) ^ (pos & m)) << 3) | (d & 7);
}

// Shared memory is a dynamic extern buffer in every kernel.
extern __shared__ __align__(16) unsigned char cmolcu_smem[];

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 128-bit streaming load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ld_nc_u32(const void *p) {
    uint32_t r;
    asm("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void *p) {
    uint16_t r;
    asm("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ld_nc_u8(const void *p) {
    uint16_t r;
    asm("ld.global.nc.u8 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Programmatic dependent launch: wait until the previous kernel in the stream
// has signalled (or finished); and allow the next one to start launching.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

#define CUDA_TRY(expr)                                                          \
    do {                                                                        \
        cudaError_t _e = (expr);                                                \
        if (_e != cudaSuccess) {                                                \
            cmolcu_set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr,         \
                             cudaGetErrorString(_e));                           \
            return -1;                                                          \
        }                                                                       \
    } while (0)

extern "C" void cmolcu_set_error(const char *fmt, ...);
