// gemm_tc.cu — batched dequant matmul on tcgen05 tensor cores (see gemm_tc.cuh).
#include "gemm_tc.cuh"
#include "gemv_launch.cuh"

#include <cuda.h>        // CUtensorMap (the encode call is reached through the runtime)
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>
#include <vector>

#define TC_DQW 8                          // dequantising warps (3..10)
#define TC_THREADS ((3 + TC_DQW) * 32)    // + weight producer warp 0, MMA warp 1, activation producer warp 2
#define TC_DQT (TC_DQW * 32)
#define TC_MAX_DEPTH 8
#define TC_TS_MIN_DEPTH 2                 // dequantised ring in tensor memory: depth range
#define TC_TS_MAX_DEPTH 4
#define TC_RU 1                           // split-K reduction: tasks per thread, and
#define TC_RS 8                           // splits of each, whose loads are in flight together

bool tc_supported(int dt) { return dt == DT_Q4_K || dt == DT_Q8_0 || dt == DT_Q4_0 || dt == DT_Q5_0; }

// ---------------------------------------------------------------------------
// tcgen05 / proxy helpers (inline PTX, sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand with the 128-byte swizzle: rows of 128 bytes (64 f16),
// 8-row groups 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);      // start address
    d |= (uint64_t)1 << 16;                        // leading byte offset (16 B; unused for this layout)
    d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset
    d |= (uint64_t)1 << 46;                        // version
    d |= (uint64_t)2 << 61;                        // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}

// The same product with A in tensor memory: row m of A is lane m, and each
// 32-bit column holds two consecutive K values (lower half first), so a K=16
// product reads 8 columns from `tmem_a`.
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                          uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t h[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3]), "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7]), "r"(h[8]), "r"(h[9]),
        "r"(h[10]), "r"(h[11]), "r"(h[12]), "r"(h[13]), "r"(h[14]), "r"(h[15])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// ---------------------------------------------------------------------------
// Activation image: one CTA per column (columns >= ncol are zero).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_tc_xprep(const float *x, long long x_ld, int K, int ncol, int npad,
                                                  const float *norm_w, float eps, uint16_t *xs) {
    pdl_wait();
    pdl_launch_dependents();
    const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float red[8];
    __shared__ float s_ir;
    const bool live = n < ncol;
    const float *xc = x + (long long)n * x_ld;
    float ir = 1.f;
    if (live && norm_w) {
        // the RMS of src/model.c:90-97, in the GEMV's summation order
        float ss = 0.f;
        for (int i = tid; i < K; i += 256) {
            const float v = xc[i];
            ss = __fmaf_rn(v, v, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
            for (int w = 0; w < 8; w++) t += red[w];
            s_ir = 1.0f / sqrtf(t / (float)K + eps);
        }
        __syncthreads();
        ir = s_ir;
    }
    // 8 consecutive values a thread per pass: two 16-byte loads of x (and of
    // the gains) when the column's start is 16-byte aligned
    const bool vec = live && ((reinterpret_cast<uintptr_t>(xc) | reinterpret_cast<uintptr_t>(norm_w)) & 15) == 0;
    for (int c = tid; c < K / 8; c += 256) {
        const int k0 = c * 8, kb = k0 >> 6, ch = (k0 & 63) >> 3;
        float v[8];
        if (vec) {
            const float4 a = *reinterpret_cast<const float4 *>(xc + k0);
            const float4 b = *reinterpret_cast<const float4 *>(xc + k0 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            if (norm_w) {
                const float4 ga = *reinterpret_cast<const float4 *>(norm_w + k0);
                const float4 gb = *reinterpret_cast<const float4 *>(norm_w + k0 + 4);
                const float g[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = __fmul_rn(g[i], __fmul_rn(v[i], ir));
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float t = live ? xc[k0 + i] : 0.f;
                if (live && norm_w) t = __fmul_rn(norm_w[k0 + i], __fmul_rn(t, ir));
                v[i] = t;
            }
        }
        uint4 o = make_uint4(pack_h2(v[0], v[1]), pack_h2(v[2], v[3]), pack_h2(v[4], v[5]), pack_h2(v[6], v[7]));
        uint4 *dst = reinterpret_cast<uint4 *>(xs + ((size_t)kb * npad + n) * 64) + (ch ^ (n & 7));
        *dst = o;
    }
}

// ---------------------------------------------------------------------------
// The matmul
// ---------------------------------------------------------------------------
#define TC_SV 256          // values per quantised slice (one K-slice of 128 rows in a stage)
#define TC_MAX_QD 4        // quantised-stage ring depth

struct TcParams {
    // per plane: the full K-chunks as a 3-D tensor (bytes of a row's chunk,
    // rows, chunk) and the last K-chunk as its own (its rows are shorter)
    CUtensorMap     tm_full[3], tm_last[3];
    GemvArgs        g;                 // weight, y, epilogue fields
    int             epi, ncol, npad;
    const uint16_t *xs;
    int             nslice;            // K-slices of the matrix (slices never cross a K-chunk)
    int             ksplit, slices_per_split;
    float          *part;
    int            *counters;
    uint32_t        tmem_cols;
    int             depth;             // A (dequantised) tile ring depth (<= TC_MAX_DEPTH)
    int             bdepth;            // B (activation) tile ring depth (<= TC_MAX_DEPTH)
    int             qdepth;            // quantised-stage ring depth (<= TC_MAX_QD)
    int             cluster;           // 1: the K splits of a row block form one cluster and add
                                       // their partials through distributed shared memory
    int             msub;              // 128-row sub-tiles per CTA (1, or 2: two TMEM accumulators
                                       // share every activation tile; no K split then)
    int             ts;                // 1: the dequantised tiles live in tensor memory (columns
                                       // a_col + (slot * msub + sub-tile) * 32 ..), not shared memory
    uint32_t        a_col;
};

// A quantised stage holds one 256-value slice of 128 rows, loaded by TMA
// tensor copies (one per plane; Q8_0's 256-byte plane-0 rows as two
// 128-byte boxes).  Plane 0 lands with the 128-byte swizzle: 16-byte chunk c
// of row r sits at chunk c ^ (r % 8) of the row's 128 bytes, so the 8 lanes
// of a shared-memory phase reading consecutive rows hit 8 bank groups.
// Planes 1 (16 bytes a row: the block scales, or Q4_K's d, dmin and 6-bit
// scales) and 2 (Q5_0's high bits, 32 bytes) are dense rows.
__host__ __device__ constexpr int tc_nb0(int dt) { return dt == DT_Q8_0 ? 2 : 1; }
__host__ __device__ constexpr int tc_p2b(int dt) { return dt == DT_Q5_0 ? 32 : 0; }
__host__ __device__ constexpr int tc_off1(int dt) { return tc_nb0(dt) * TC_M * 128; }
__host__ __device__ constexpr int tc_off2(int dt) { return tc_off1(dt) + TC_M * 16; }
__host__ __device__ constexpr int tc_stage_tx(int dt) { return tc_off2(dt) + TC_M * tc_p2b(dt); }
__host__ __device__ constexpr int tc_stage_bytes(int dt) { return (tc_stage_tx(dt) + 1023) / 1024 * 1024; }

// The 16 bytes at byte `bo` of row r's plane-0 slice.
__device__ __forceinline__ const uint8_t *tc_q0(const uint8_t *st, int r, int bo) {
    return st + (bo >> 7) * (TC_M * 128) + r * 128 + ((((bo >> 4) & 7) ^ (r & 7)) << 4);
}

// Slice t of the matrix: K-chunk j, value offset `off` in it, `len` values.
__host__ __device__ inline void tc_slice(const QWeight &w, int t, int &j, int &off, int &len) {
    const int spc = w.kc / TC_SV;                      // slices of a full K-chunk (kc is a multiple of 256 if nkc > 1)
    const int full = (w.nkc - 1) * spc;
    if (t < full) {
        j = t / spc;
        off = (t % spc) * TC_SV;
        len = TC_SV;
    } else {
        j = w.nkc - 1;
        off = (t - full) * TC_SV;
        len = min(TC_SV, qw_chunk_values(w, j) - off);
    }
}

// 32 dequantised values of row r, values [v, v + 32) of the slice held in
// the quantised stage (v a multiple of 32: one Q8_0 / Q4_0 / Q5_0 block, or
// one 32-value group of a Q4_K super-block; GGUF block arithmetic of
// src/quant.c:152-194), as 16 packed f16 pairs.  No conversion
// instructions: a small unsigned integer u becomes the f16 1024 + u by
// placing it under the exponent bits 0x6400 (one byte permute per pair), and
// the f32 2^23 + u under 0x4B000000.
//   Q8_0, Q4_0, Q5_0: q is exact in f16 and the block scale d is an f16, so
//                     (1024 + u - bias) * d in f16 arithmetic is the f16
//                     rounding of the exact value d * q.
//   Q4_K:             d * sc * q - dmin * mn in f32 (sc, mn 6-bit; pairs of
//                     values in packed f32x2 arithmetic), then f16.
__device__ __forceinline__ uint32_t h2_from_bytes(uint32_t w, uint32_t sel) {
    // bytes of w selected by sel into the low byte of each half, 0x64 above
    return __byte_perm(w, 0x64646464u, sel);
}

// f16 pair of a * q - m for the two f32 patterns 2^23 + q in b0, b1
// (a2 = {a, a}, nm2 = {-m, -m}): the exact subtraction of 2^23, one fused
// multiply-add per value, one rounding to f16.
__device__ __forceinline__ uint32_t q4k_h2(uint32_t b0, uint32_t b1, uint64_t a2, uint64_t nm2) {
    const uint64_t n23 = 0xCB000000CB000000ull;   // {-2^23, -2^23}
    uint64_t v, r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(b0), "r"(b1));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(v) : "l"(v), "l"(n23));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(v), "l"(a2), "l"(nm2));
    uint32_t lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(r));
    return pack_h2(__uint_as_float(lo), __uint_as_float(hi));
}

template <int DT>
__device__ __forceinline__ void tc_dequant32(const uint8_t *st, int r, int v, uint32_t out[16]) {
    const uint8_t *P1 = st + tc_off1(DT) + r * 16, *P2 = st + tc_off2(DT) + r * tc_p2b(DT);
    if constexpr (DT == DT_Q4_K) {
        // one super-block per slice: v in [0, 256); values v.. of pair pj,
        // low nibbles for the pair's first 32 values, high for the second
        const int pj = v >> 6, half = (v >> 5) & 1;
        const uint4 p0 = *reinterpret_cast<const uint4 *>(tc_q0(st, r, 32 * pj));
        const uint4 p1 = *reinterpret_cast<const uint4 *>(tc_q0(st, r, 32 * pj + 16));
        const uint4 h = *reinterpret_cast<const uint4 *>(P1);
        const float d = h2f((uint16_t)(h.x & 0xFFFF)), dmin = h2f((uint16_t)(h.x >> 16));
        float sc0, sc1, mn0, mn1;
        q4k_pair(h.y, h.z, h.w, pj, sc0, sc1, mn0, mn1);
        const float a = d * (half ? sc1 : sc0), m = dmin * (half ? mn1 : mn0);
        uint64_t a2, nm2;
        asm("mov.b64 %0, {%1, %1};" : "=l"(a2) : "f"(a));
        asm("mov.b64 %0, {%1, %1};" : "=l"(nm2) : "f"(-m));
        const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t t = half ? ((w[i] >> 4) & 0x0F0F0F0Fu) : (w[i] & 0x0F0F0F0Fu);
            out[2 * i] = q4k_h2(__byte_perm(t, 0x4B000000u, 0x7540u), __byte_perm(t, 0x4B000000u, 0x7541u), a2, nm2);
            out[2 * i + 1] = q4k_h2(__byte_perm(t, 0x4B000000u, 0x7542u), __byte_perm(t, 0x4B000000u, 0x7543u), a2, nm2);
        }
    } else {
        const int b = v >> 5;
        uint32_t w[8];
        __half bias;
        const __half d = __ushort_as_half(*reinterpret_cast<const uint16_t *>(P1 + b * 2));
        if constexpr (DT == DT_Q8_0) {
            const uint4 p0 = *reinterpret_cast<const uint4 *>(tc_q0(st, r, b * 32));
            const uint4 p1 = *reinterpret_cast<const uint4 *>(tc_q0(st, r, b * 32 + 16));
            const uint32_t raw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) w[i] = raw[i] ^ 0x80808080u;   // int8 -> unsigned + 128
            bias = __ushort_as_half((uint16_t)0x6480);                  // 1024 + 128
        } else {
            // 16 bytes: value i in the low nibble of byte i, value 16 + i in the high
            const uint4 pl = *reinterpret_cast<const uint4 *>(tc_q0(st, r, b * 16));
            const uint32_t raw[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                w[i] = raw[i] & 0x0F0F0F0Fu;
                w[4 + i] = (raw[i] >> 4) & 0x0F0F0F0Fu;
            }
            if constexpr (DT == DT_Q5_0) {
                const uint32_t qh = *reinterpret_cast<const uint32_t *>(P2 + b * 4);
#pragma unroll
                for (int i = 0; i < 8; i++) w[i] |= spread4_bit4((qh >> (4 * i)) & 15u);
                bias = __ushort_as_half((uint16_t)0x6410);              // 1024 + 16
            } else {
                bias = __ushort_as_half((uint16_t)0x6408);              // 1024 + 8
            }
        }
        const __half2 b2 = __halves2half2(bias, bias), d2 = __halves2half2(d, d);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t lo = h2_from_bytes(w[i], 0x5140u), hi = h2_from_bytes(w[i], 0x5342u);
            __half2 x0 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&lo), b2), d2);
            __half2 x1 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&hi), b2), d2);
            out[2 * i] = *reinterpret_cast<const uint32_t *>(&x0);
            out[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&x1);
        }
    }
}

// TMA tensor copy of one box at (x, y, z) of `map` into shared memory,
// completing in bytes on `bar` (no multicast).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Distributed shared memory: the address of shared offset `saddr` in the
// cluster's CTA `rank`, a 16-byte load from it, and the cluster-wide barrier
// (release / acquire: shared-memory writes before it are visible to every
// CTA of the cluster after it).
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Epilogue of one value (STORE, RESID) or of a row pair (SWIGLU, QKV; the
// even row's thread writes).
__device__ __forceinline__ void tc_epilogue(const TcParams &p, int row, int col, float v, float partner) {
    const GemvArgs &g = p.g;
    if (row >= g.w.rows || col >= p.ncol) return;
    switch (p.epi) {
    case EPI_STORE:
        g.y[(long long)col * g.y_ld + row] = v;
        break;
    case EPI_RESID: {
        float *y = g.y + (long long)col * g.y_ld + row;
        *y = __ldcg(y) + v;
        break;
    }
    case EPI_SWIGLU:
        if (!(row & 1) && row + 1 < g.w.rows) epi_swiglu_pair(g, row, col, v, partner);
        break;
    default:
        if (!(row & 1) && row + 1 < g.w.rows) epi_qkv_pair(g, row, col, v, partner);
        break;
    }
}

// Adds the split partials of this row block for columns [c_lo, c_hi) and
// runs the epilogue.  Task = (column, 4 consecutive rows); a thread takes
// TC_RU tasks at once and loads TC_RS splits of each before adding any, so
// TC_RU * TC_RS float4 loads are in flight together (the partials come from
// other CTAs' shared memory or from L2: latency, not bandwidth, bounds this).
// Partials add in split order (deterministic); the even row of a pair
// applies pair epilogues.  load(split, column, row quad) -> float4.
template <typename LoadF>
__device__ __forceinline__ void tc_reduce_cols(const TcParams &p, int m0, int c_lo, int c_hi, int tid, LoadF load) {
    constexpr int RQ = TC_M / 4;
    const int ntask = RQ * max(0, c_hi - c_lo);
    for (int base = tid; base < ntask; base += TC_RU * TC_THREADS) {
        float4 acc[TC_RU];
#pragma unroll
        for (int u = 0; u < TC_RU; u++) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < p.ksplit; s0 += TC_RS) {
            float4 v[TC_RU][TC_RS];
#pragma unroll
            for (int u = 0; u < TC_RU; u++) {
                const int idx = base + u * TC_THREADS;
#pragma unroll
                for (int r = 0; r < TC_RS; r++)
                    v[u][r] = idx < ntask && s0 + r < p.ksplit ? load(s0 + r, c_lo + idx / RQ, idx % RQ)
                                                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < TC_RU; u++)
#pragma unroll
                for (int r = 0; r < TC_RS; r++) {
                    acc[u].x += v[u][r].x; acc[u].y += v[u][r].y; acc[u].z += v[u][r].z; acc[u].w += v[u][r].w;
                }
        }
#pragma unroll
        for (int u = 0; u < TC_RU; u++) {
            const int idx = base + u * TC_THREADS;
            if (idx >= ntask) continue;
            const int col = c_lo + idx / RQ, row = m0 + 4 * (idx % RQ);
            const float a4[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                if (p.epi == EPI_STORE || p.epi == EPI_RESID) {
                    tc_epilogue(p, row + e, col, a4[e], a4[e + 1]);
                    tc_epilogue(p, row + e + 1, col, a4[e + 1], a4[e]);
                } else {
                    tc_epilogue(p, row + e, col, a4[e], a4[e + 1]);
                }
            }
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(TC_THREADS, 2) k_tc_gemm(const __grid_constant__ TcParams p) {
    const QWeight &w = p.g.w;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = blockIdx.x, ks = blockIdx.y;
    const int MS = p.msub;
    const int m0 = rb * TC_M * MS;
    const int npad = p.npad;
    const int s0 = ks * p.slices_per_split, s1 = min(p.nslice, s0 + p.slices_per_split);
    constexpr int QB = tc_stage_bytes(DT);                   // one 128-row sub-tile of a slice

    // shared memory: A tiles, B tiles (1024-aligned), quantised stages, barriers
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)cmolcu_smem + 1023) & ~(uintptr_t)1023);
    const int D = p.depth, DB = p.bdepth, QD = p.qdepth;
    uint8_t *A = base;                                        // D x MS x 16 KB (none in tensor memory)
    uint8_t *B = A + (p.ts ? (size_t)0 : (size_t)D * MS * TC_M * 128);   // DB x npad * 128
    uint8_t *Q = B + (size_t)DB * npad * 128;                 // QD x MS x QB
    uint64_t *bars = reinterpret_cast<uint64_t *>(Q + (size_t)QD * MS * QB);
    uint64_t *accfull = bars, *qfull = bars + 1, *qempty = qfull + TC_MAX_QD, *afull = qempty + TC_MAX_QD,
             *aempty = afull + TC_MAX_DEPTH, *bfull = aempty + TC_MAX_DEPTH, *bempty = bfull + TC_MAX_DEPTH;
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;
    // Set when a bounded wait of any role ran out (the fault word holds the
    // code): no role starts new copies or products after it, and each
    // producer waits for the copies it has issued before the CTA tears down.
    __shared__ int s_abort;
    volatile int *abort_flag = &s_abort;

    if (tid == 0) {
        // the weight's tensor maps, fetched while the rest of the setup runs
#pragma unroll
        for (int pl = 0; pl < (DT == DT_Q5_0 ? 3 : 2); pl++) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_last[pl])) : "memory");
            if (w.nkc > 1)
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_full[pl])) : "memory");
        }
        for (int i = 0; i < QD; i++) {
            mbar_init(&qfull[i], 1);        // the producer's arrival with the stage's byte count
            mbar_init(&qempty[i], TC_DQW);
        }
        for (int i = 0; i < D; i++) {
            mbar_init(&afull[i], TC_DQW);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < DB; i++) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        mbar_init(accfull, 1);
        fence_mbar_init();
        s_abort = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_launch_dependents();

    // k-blocks of this CTA (every slice holds a whole number of them)
    int nkb = 0;
    for (int t = s0; t < s1; t++) {
        int j, off, len;
        tc_slice(w, t, j, off, len);
        nkb += len / TC_KB;
    }

    if (warp == 0) {
        // ---------------- weight producer: one TMA copy per plane and slice ----------------
        // gated only by the dequantising warps releasing stages, so the ring
        // runs QD slices ahead of the dequantisation
        if (lane == 0) {
            int issued = 0;
            for (int t = s0; t < s1; t++) {
                const int li = t - s0, stg = li % QD, use = li / QD;
                if (*abort_flag) break;
                if (use > 0 && !mbar_wait(&qempty[stg], (use - 1) & 1, p.g.fault, FAULT_GEMV_EMPTY)) {
                    *abort_flag = 1;
                    break;
                }
                int j, off, len;
                tc_slice(w, t, j, off, len);
                const bool last = j == w.nkc - 1;
                const CUtensorMap *mp = last ? p.tm_last : p.tm_full;
                const int z = last ? 0 : j;
                const int o0 = qw_plane_bytes(DT, 0, off), o1 = qw_plane_bytes(DT, 1, off);
                mbar_arrive_expect_tx(&qfull[stg], (uint32_t)(MS * tc_stage_tx(DT)));
                for (int sb = 0; sb < MS; sb++) {
                    uint8_t *q = Q + ((size_t)stg * MS + sb) * QB;
                    const int my = m0 + TC_M * sb;
#pragma unroll
                    for (int b = 0; b < tc_nb0(DT); b++)
                        tma_load_3d(q + b * TC_M * 128, &mp[0], o0 + 128 * b, my, z, &qfull[stg]);
                    tma_load_3d(q + tc_off1(DT), &mp[1], o1, my, z, &qfull[stg]);
                    if constexpr (DT == DT_Q5_0)
                        tma_load_3d(q + tc_off2(DT), &mp[2], qw_plane_bytes(DT, 2, off), my, z, &qfull[stg]);
                }
                issued = li + 1;
            }
            // the last QD slices issued have landed before the CTA goes on
            // (immediately true for the ones the dequantisation consumed)
            for (int li = issued - 1; li >= 0 && li >= issued - QD; li--)
                mbar_wait(&qfull[li % QD], (li / QD) & 1, nullptr, 0);
        }
    } else if (warp == 2) {
        // ---------------- activation producer: one k-block of the image per tile slot ----------------
        if (lane == 0) {
            pdl_wait();   // the activation image comes from the previous kernel
            int bn = 0, slot = 0, u = 0;                // tiles issued; ring slot and its use
            bool ok = true;
            for (int t = s0; t < s1 && ok; t++) {
                int j, off, len;
                tc_slice(w, t, j, off, len);
                const int g0 = (j * w.kc + off) / TC_KB;
                for (int i = 0; i < len / TC_KB; i++, bn++, u += ++slot == DB, slot = slot == DB ? 0 : slot) {
                    if (*abort_flag) { ok = false; break; }
                    if (u > 0 && !mbar_wait(&bempty[slot], (u - 1) & 1, p.g.fault, FAULT_GEMV_EMPTY)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&bfull[slot], (uint32_t)(npad * 128));
                    bulk_g2s(B + (size_t)slot * npad * 128, p.xs + (size_t)(g0 + i) * npad * 64, (uint32_t)(npad * 128),
                             &bfull[slot]);
                }
            }
            for (int b = bn - 1; b >= 0 && b >= bn - DB; b--)   // the copies issued have landed
                mbar_wait(&bfull[b % DB], (b / DB) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(npad >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
            // ring slots and their parities advance by counting (no division in the loop)
            int slot = 0, use = 0, bslot = 0, buse = 0;
            for (int i = 0; i < nkb; i++, use += ++slot == D, slot = slot == D ? 0 : slot,
                     buse += ++bslot == DB, bslot = bslot == DB ? 0 : bslot) {
                if (*abort_flag || !mbar_wait(&afull[slot], use & 1, p.g.fault, FAULT_GEMV_FULL) ||
                    !mbar_wait(&bfull[bslot], buse & 1, p.g.fault, FAULT_GEMV_FULL)) {
                    *abort_flag = 1;
                    break;                              // accfull below still tracks the products issued
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(A + (size_t)slot * MS * TC_M * 128);
                const uint32_t b_addr = smem_u32(B + (size_t)bslot * npad * 128);
                for (int sb = 0; sb < MS; sb++) {        // sub-tile sb accumulates at columns [sb * npad, ...)
                    if (p.ts) {
                        const uint32_t ta = tmem + p.a_col + (uint32_t)((slot * MS + sb) * 32);
#pragma unroll
                        for (int k = 0; k < TC_KB / 16; k++)
                            tc_mma_ts(tmem + (uint32_t)(sb * npad), ta + 8 * k, tc_desc(b_addr + 32 * k), idesc,
                                      (i | k) != 0);
                    } else {
#pragma unroll
                        for (int k = 0; k < TC_KB / 16; k++)
                            tc_mma(tmem + (uint32_t)(sb * npad), tc_desc(a_addr + sb * TC_M * 128 + 32 * k),
                                   tc_desc(b_addr + 32 * k), idesc, (i | k) != 0);
                    }
                }
                tc_commit(&aempty[slot]);
                tc_commit(&bempty[bslot]);
            }
            tc_commit(accfull);
        }
    } else {
        // ---------------- dequantise ----------------
        const int dt = tid - 96;
        int i = 0, slot = 0, use = 0;                   // k-blocks done; A ring slot and its use
        bool dq_ok = true;
        for (int t = s0; t < s1 && dq_ok; t++) {
            const int li = t - s0, stg = li % QD;
            // warp-uniform outcome of each wait: the warp leaves its loops together
            if (!__all_sync(0xffffffffu, !*abort_flag && mbar_wait(&qfull[stg], (li / QD) & 1, p.g.fault,
                                                                             FAULT_GEMV_FULL))) {
                *abort_flag = 1;
                break;
            }
            int j, off, len;
            tc_slice(w, t, j, off, len);
            for (int ib = 0; ib < len / TC_KB; ib++, i++, use += ++slot == D, slot = slot == D ? 0 : slot) {
                if (use > 0 && !__all_sync(0xffffffffu, mbar_wait(&aempty[slot], (use - 1) & 1, p.g.fault,
                                                                        FAULT_GEMV_EMPTY))) {
                    *abort_flag = 1;
                    dq_ok = false;
                    break;
                }
                // task = (row r, 32-value half hf): 128 rows x 2 halves a sub-tile, one per thread
                static_assert(TC_M * 2 == TC_DQT, "one 32-value task per dequantising thread");
                if (p.ts) {
                    // warp w writes tensor-memory lanes 32 * (w % 4) ..: row = that lane,
                    // warps 3-6 the first 32 values of the k-block, warps 7-10 the second
                    const int quarter = warp & 3, r = 32 * quarter + lane, hf = (warp - 3) >> 2;
                    for (int sb = 0; sb < MS; sb++) {
                        uint32_t h[16];
                        tc_dequant32<DT>(Q + ((size_t)stg * MS + sb) * QB, r, ib * TC_KB + 32 * hf, h);
                        tc_st16(tmem + ((uint32_t)(32 * quarter) << 16) + p.a_col +
                                    (uint32_t)((slot * MS + sb) * 32 + 16 * hf),
                                h);
                    }
                    tc_wait_st();
                    tc_fence_before();   // the tensor core reads the tile after the barrier
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[slot]);
                    continue;
                }
                for (int sb = 0; sb < MS; sb++) {
                    const uint8_t *q = Q + ((size_t)stg * MS + sb) * QB;
                    uint8_t *tile = A + ((size_t)slot * MS + sb) * TC_M * 128;
                    const int r = dt >> 1, hf = dt & 1;
                    uint32_t h[16];
                    tc_dequant32<DT>(q, r, ib * TC_KB + 32 * hf, h);
                    uint4 *row = reinterpret_cast<uint4 *>(tile + r * 128);
#pragma unroll
                    for (int c = 0; c < 4; c++)
                        row[(4 * hf + c) ^ (r & 7)] = make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
                }
                fence_proxy_async_smem();   // the tensor core reads the tile through the async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[slot]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&qempty[stg]);
        }
        // ---------------- epilogue: tensor memory -> registers ----------------
        // The 8 dequantising warps: warp w reads TMEM lanes 32 * (w % 4) ..;
        // warps 3-6 and 7-10 take the two sub-tiles (MS = 2) or the two
        // halves of the columns (MS = 1).
        {
            const int ew = warp - 3, quarter = warp & 3, grp = ew >> 2;
            const int sb = MS == 2 ? grp : 0;
            const int ch = npad >= 32 ? (npad / 32) * 16 : npad;    // column split of MS = 1 (16-column units)
            const int c_lo = MS == 2 ? 0 : (grp ? ch : 0), c_hi = MS == 2 ? npad : (grp ? npad : ch);
            const int row = m0 + TC_M * sb + 32 * quarter + lane;
            mbar_wait(accfull, 0, p.g.fault, FAULT_GEMV_FULL);
            tc_fence_after();
            if (p.ksplit == 1) pdl_wait();
            for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                float v[16];
                tc_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(sb * npad + c0), v);
                if (p.ksplit == 1 && p.epi == EPI_SWIGLU) {
                    // rows (2j, 2j + 1) are (gate, up) of output j, held by a lane
                    // pair: the even lane finishes the even columns, the odd lane
                    // the odd ones (each lane sends the partner the value it lacks)
                    const bool odd = lane & 1;
                    const int pr = row & ~1;
#pragma unroll
                    for (int e = 0; e < 16; e += 2) {
                        const float got = __shfl_xor_sync(0xffffffffu, odd ? v[e] : v[e + 1], 1);
                        const int col = c0 + e + (odd ? 1 : 0);
                        if (pr + 1 < p.g.w.rows && col < p.ncol)
                            epi_swiglu_pair(p.g, pr, col, odd ? got : v[e], odd ? v[e + 1] : got);
                    }
                } else if (p.ksplit == 1) {
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 1);
                        tc_epilogue(p, row, c0 + e, v[e], partner);
                    }
                } else {
                    // partial sums: [column][row] in this CTA's shared memory (the
                    // rings are drained: every copy and MMA has completed) or in
                    // global scratch
                    float *pp = p.cluster ? reinterpret_cast<float *>(base) + (size_t)c0 * TC_M + (row - m0)
                                          : p.part + ((size_t)(rb * p.ksplit + ks) * npad + c0) * TC_M + (row - m0);
#pragma unroll
                    for (int e = 0; e < 16; e++) pp[(size_t)e * TC_M] = v[e];
                }
            }
        }
    }

    // ---------------- split-K: the partials of the row block's K splits are added ----------------
    // The roles above leave warps 0-2 diverged (lane 0 ran the loops); the
    // CTA barrier counts whole warps, so each warp re-converges first.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (p.ksplit > 1 && p.cluster) {
        // every CTA of the cluster has its partial in shared memory; CTA s adds
        // columns [s * cw, (s + 1) * cw) over the cluster, in split order
        cluster_sync_all();
        pdl_wait();
        const int cw = (npad + p.ksplit - 1) / p.ksplit;
        const int c_lo = ks * cw, c_hi = min(npad, c_lo + cw);
        const uint32_t ps = smem_u32(base);
        tc_reduce_cols(p, m0, c_lo, c_hi, tid, [&](int sp, int col, int rq) {
            return ld_dsmem_f4(dsmem_addr(ps + (uint32_t)((col * TC_M + 4 * rq) * 4), (uint32_t)sp));
        });
        cluster_sync_all();   // the partials stay in place until every CTA has read them
    } else if (p.ksplit > 1) {
        // the last CTA of the row block (atomic counter) adds the global partials
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&p.counters[rb], 1) == p.ksplit - 1;
        __syncwarp();
        __syncthreads();
        if (s_last) {
            __threadfence();
            pdl_wait();
            const float4 *P4 = reinterpret_cast<const float4 *>(p.part);
            tc_reduce_cols(p, m0, 0, npad, tid, [&](int sp, int col, int rq) {
                return __ldcg(P4 + (((size_t)(rb * p.ksplit + sp) * npad + col) * TC_M) / 4 + rq);
            });
            if (tid == 0) p.counters[rb] = 0;
        }
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int tc_npad(int ncol) { return std::max(16, (ncol + 15) / 16 * 16); }

// Ring depths and shared memory of one CTA: two CTAs share an SM when both
// fit (<= 112 KB each, narrow batches); otherwise one CTA takes the SM and
// deeper rings.
// Tuning knobs read once per process (measurements): CMOLCU_TC_PER_SM=1
// forces one CTA per SM, CMOLCU_TC_KSPLIT_MAX caps the split of K.
static int tc_knob(const char *name, int dflt) {
    const char *v = getenv(name);
    return v && *v ? atoi(v) : dflt;
}

// Ring depths and shared memory of one CTA.  Two CTAs share an SM when the
// minimum rings fit in ~112 KB (narrow batches); otherwise one CTA takes the
// SM.  Spare room deepens, in this order: the activation ring (its tiles
// are small at narrow batches, and a shallow one puts an L2 round trip
// behind every k-block's MMA), the dequantised ring, the quantised ring.
// With `ts` the dequantised ring lives in tensor memory (no shared memory;
// its depth is set by the caller).
static void tc_rings(int dt, int npad, int ms, bool ts, int &depth, int &bdepth, int &qdepth, size_t &smem,
                     int &per_sm) {
    static const int max_per_sm = tc_knob("CMOLCU_TC_PER_SM", 2) == 1 ? 1 : 2;
    const size_t qb = (size_t)ms * tc_stage_bytes(dt), bars = (1 + 2 * TC_MAX_QD + 4 * TC_MAX_DEPTH) * 8;
    const size_t a_slot = ts ? 0 : (size_t)ms * TC_M * 128, b_slot = (size_t)npad * 128;
    auto need = [&](int da, int db, int dq) { return 1024 + da * a_slot + db * b_slot + dq * qb + bars; };
    // CMOLCU_TC_RINGS="A,B,Q": ring depths for steps of more than 64 columns
    // (measurements), used when they fit one CTA per SM
    static const char *rings = getenv("CMOLCU_TC_RINGS");
    int fa = 0, fb = 0, fq = 0;
    if (rings && npad > 64 && sscanf(rings, "%d,%d,%d", &fa, &fb, &fq) == 3 && fa >= 2 && fa <= TC_MAX_DEPTH &&
        fb >= 2 && fb <= TC_MAX_DEPTH && fq >= 2 && fq <= TC_MAX_QD && need(fa, fb, fq) <= 220 * 1024) {
        depth = fa; bdepth = fb; qdepth = fq; per_sm = 1;
        smem = need(fa, fb, fq);
        return;
    }
    for (per_sm = ts ? 1 : max_per_sm; per_sm >= 1; per_sm--) {   // tensor-memory tiles need the whole TMEM
        const size_t budget = per_sm == 2 ? 112 * 1024 : 220 * 1024;
        depth = bdepth = qdepth = 2;
        if (need(2, 2, 2) > budget && per_sm == 2) continue;
        const int steps[][3] = {{0, 4, 0}, {3, 0, 0}, {0, 0, 3}, {0, 8, 0}, {4, 0, 0}, {0, 0, 4}};
        for (const auto &st : steps) {
            const int da = std::max(depth, st[0]), db = std::max(bdepth, st[1]), dq = std::max(qdepth, st[2]);
            for (int b = db; b >= bdepth; b--)     // as deep a B ring as fits at this step
                if (need(da, b, dq) <= budget) {
                    depth = da; bdepth = b; qdepth = dq;
                    break;
                }
        }
        smem = need(depth, bdepth, qdepth);
        return;
    }
    per_sm = 1;
    depth = bdepth = qdepth = 2;
    smem = need(2, 2, 2);
}

static int tc_nslice(int k, int kc) {
    const int nkc = (k + kc - 1) / kc;
    const int last = k - (nkc - 1) * kc;
    return (nkc - 1) * (kc / TC_SV) + (last + TC_SV - 1) / TC_SV;
}

// K split of a row block: as many splits as fill one wave of CTAs, at most
// TC_WIDE_KSPLIT of them at steps of 128 columns or more.  There each split's
// partial is npad x 128 floats and the reduction's cost grows with the number
// of splits faster than the extra SMs pay back: at 256 columns, capping the
// split at 6 took 2048 x 11008 from 60.3 to 43.6 us and 2048 x 2048 from 28.6
// to 18.9 us (graph replay; caps 2, 3 and 4 measured slower than 6); at 128
// columns 2048 x 11008 from 44.2 to 37.3 us.  At 32 and 64 columns the cap
// measured no better.
#define TC_WIDE_KSPLIT 6
static void tc_split(int rows, int nslice, int per_sm, int ms, int npad, int &rblocks, int &ksplit, int &sps) {
    static const int knob = tc_knob("CMOLCU_TC_KSPLIT_MAX", 0);
    const int cap = knob > 0 ? knob : npad >= 128 ? TC_WIDE_KSPLIT : 1 << 20;
    const int slots = device_sm_count() * per_sm;
    rblocks = (rows + TC_M * ms - 1) / (TC_M * ms);
    ksplit = ms > 1 ? 1 : std::max(1, std::min(std::min(nslice, cap), slots / rblocks));    // one wave
    sps = (nslice + ksplit - 1) / ksplit;
    ksplit = (nslice + sps - 1) / sps;
}

void tc_scratch_need(int rows, int k, int ncol, size_t *xs_halves, size_t *part_floats, int *row_blocks) {
    const int npad = tc_npad(ncol);
    *xs_halves = (size_t)k * npad;
    int rb, ks, sps;
    tc_split(rows, k / TC_KB, 2, 1, 16, rb, ks, sps);   // an upper bound on the split of any format and width
    *part_floats = ks > 1 ? (size_t)rb * ks * npad * TC_M : 0;
    *row_blocks = rb;
}

typedef void (*tc_kernel_t)(TcParams);

#define TC_MAX_CLUSTER 16    // K splits of a row block that may form one cluster (8 portable)

// True when `ks` CTAs of `smem` bytes can run as one (1, ks, 1) cluster of
// kernel k on this device (cached per kernel, size and device).
static bool tc_cluster_ok(tc_kernel_t k, int ks, int rb, size_t smem) {
    struct Entry { tc_kernel_t k; int ks, dev; size_t smem; bool ok; };
    static std::vector<Entry> cache;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    for (const Entry &e : cache)
        if (e.k == k && e.ks == ks && e.dev == dev && e.smem == smem) return e.ok;
    bool ok = ks >= 2 && ks <= TC_MAX_CLUSTER;
    if (ok && ks > 8 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        ok = false;
    if (ok) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(rb, ks);
        cfg.blockDim = dim3(TC_THREADS);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = ks;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        ok = cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess && n >= 1;
    }
    cudaGetLastError();   // a refused query leaves no sticky error
    cache.push_back({k, ks, dev, smem, ok});
    return ok;
}

// The matmul launch: PDL, and a (1, cluster_y, 1) cluster when cluster_y > 1.
static cudaError_t tc_launch(tc_kernel_t k, dim3 grid, size_t smem, cudaStream_t st, bool pdl, int cluster_y,
                             const TcParams &p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (cluster_y > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = 1;
        at[na].val.clusterDim.y = cluster_y;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, p);
}

// cuTensorMapEncodeTiled, reached through the runtime's driver entry point
// (no link-time dependency on the driver library).
typedef CUresult (*tc_encode_t)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static tc_encode_t tc_encode_fn() {
    static const tc_encode_t fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<tc_encode_t>(f);
    }();
    return fn;
}

// Tensor map of one plane: x = bytes of a row's K-chunk (16-byte multiple),
// y = rows, z = K-chunks (`nz`, each rows * row_bytes apart); box
// box_x bytes x 128 rows x 1, with the 128-byte swizzle for plane 0.  Boxes
// reaching past the rows or a short chunk read zeros.
static bool tc_plane_map(CUtensorMap *m, const uint8_t *base, int row_bytes, int rows, int nz, int box_x, bool swz) {
    const tc_encode_t enc = tc_encode_fn();
    if (!enc || row_bytes <= 0 || rows <= 0 || nz <= 0) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)rows, (cuuint64_t)nz};
    const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)row_bytes * (cuuint64_t)rows};
    const cuuint32_t box[3] = {(cuuint32_t)box_x, (cuuint32_t)TC_M, 1u};
    const cuuint32_t es[3] = {1u, 1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The full-chunk and last-chunk maps of every plane the format has.
static bool tc_weight_maps(const QWeight &w, TcParams &p) {
    const int np = w.dtype == DT_Q5_0 ? 3 : 2;
    for (int pl = 0; pl < np; pl++) {
        const int box = pl == 0 ? 128 : pl == 1 ? 16 : 32;
        if (w.nkc > 1 && !tc_plane_map(&p.tm_full[pl], w.p[pl], w.cs[pl], w.prow, w.nkc - 1, box, pl == 0))
            return false;
        const uint8_t *last = w.p[pl] + (size_t)(w.nkc - 1) * w.prow * w.cs[pl];
        if (!tc_plane_map(&p.tm_last[pl], last, w.cl[pl], w.prow, 1, box, pl == 0)) return false;
    }
    return true;
}

static tc_kernel_t tc_pick(int dt) {
    switch (dt) {
    case DT_Q4_K: return k_tc_gemm<DT_Q4_K>;
    case DT_Q8_0: return k_tc_gemm<DT_Q8_0>;
    case DT_Q4_0: return k_tc_gemm<DT_Q4_0>;
    case DT_Q5_0: return k_tc_gemm<DT_Q5_0>;
    default: return nullptr;
    }
}

cudaError_t tc_matmul(const GemvArgs &a, int ncol, int epi, const TcScratch &s, cudaStream_t st, bool pdl) {
    const QWeight &w = a.w;
    tc_kernel_t k = tc_pick(w.dtype);
    if (!k || ncol < 1 || ncol > TC_MAX_N || w.k % TC_KB || a.x_inc != 1 || a.y_inc != 1) return cudaErrorInvalidValue;
    if (w.nkc > 1 && w.kc % TC_SV) return cudaErrorInvalidValue;
    if (w.dtype == DT_Q4_K && w.k % TC_SV) return cudaErrorInvalidValue;
    const int npad = tc_npad(ncol);
    // Two 128-row sub-tiles per CTA (both accumulators reuse every activation
    // tile, halving its shared-memory ingest per output row) for wide steps
    // on matrices with rows for well over half a wave of such CTAs, when the
    // rings still fit (not Q8_0, whose slices are twice as large).
    // CMOLCU_TC_TS=1: the dequantised tiles go to tensor memory beside the
    // accumulators when a ring of at least TC_TS_MIN_DEPTH of them fits in the
    // 512 columns (one CTA an SM) at steps wider than 128 columns, so the
    // tensor core reads only the activation tiles from shared memory (one
    // 128-row sub-tile then).  Off by default: measured on the config-4
    // shapes at 256 columns it ties the shared-memory form on the split-K
    // matrices and loses on the 22016-row one, whose two-sub-tile CTAs it
    // cannot hold (2 x 256 accumulator columns fill the tensor memory).
    static const int ms_knob = tc_knob("CMOLCU_TC_MSUB", 0);
    static const bool ts_on = tc_knob("CMOLCU_TC_TS", 0) != 0;
    int ms = (npad >= 128 && w.rows >= 2 * TC_M * 64 && w.dtype != DT_Q8_0) ? 2 : 1;
    if (ts_on && npad > 128) ms = 1;
    if (ms_knob == 1 || ms_knob == 2) ms = ms_knob;
    int depth, bdepth, qdepth, per_sm;
    size_t smem;
    auto ts_acol = [&](int m) { return (m * npad + 31) / 32 * 32; };   // the ring starts on a 32-column boundary
    auto ts_depth = [&](int m) { return std::min(TC_TS_MAX_DEPTH, (512 - ts_acol(m)) / (m * 32)); };
    bool ts = ts_on && npad > 128 && ts_depth(ms) >= TC_TS_MIN_DEPTH;
    tc_rings(w.dtype, npad, ms, ts, depth, bdepth, qdepth, smem, per_sm);
    if (ms == 2 && smem > 220 * 1024) {
        ms = 1;
        ts = ts_on && npad > 128 && ts_depth(ms) >= TC_TS_MIN_DEPTH;
        tc_rings(w.dtype, npad, ms, ts, depth, bdepth, qdepth, smem, per_sm);
    }
    if (ts) depth = ts_depth(ms);
    const int nslice = tc_nslice(w.k, w.kc);
    int rb, ks, sps;
    tc_split(w.rows, nslice, per_sm, ms, npad, rb, ks, sps);
    if (!s.xs || rb > s.max_row_blocks || (ks > 1 && (size_t)rb * ks * npad * TC_M > s.part_floats))
        return cudaErrorInvalidValue;
    TcParams p = {};
    p.g = a;
    p.g.ncol = ncol;
    p.epi = epi;
    p.ncol = ncol;
    p.npad = npad;
    p.xs = s.xs;
    p.nslice = nslice;
    p.ksplit = ks;
    p.slices_per_split = sps;
    p.part = s.part;
    p.counters = s.counters;
    p.msub = ms;
    p.ts = ts ? 1 : 0;
    p.a_col = (uint32_t)ts_acol(ms);
    const int tcols = ts ? ts_acol(ms) + depth * ms * 32 : ms * npad;
    p.tmem_cols = tcols <= 32 ? 32 : tcols <= 64 ? 64 : tcols <= 128 ? 128 : tcols <= 256 ? 256 : 512;
    p.depth = depth;
    p.bdepth = bdepth;
    p.qdepth = qdepth;
    if (!tc_weight_maps(w, p)) return cudaErrorInvalidValue;
    static size_t attr_done[64][4];
    int dev = 0;
    cudaGetDevice(&dev);
    const int di = w.dtype == DT_Q4_K ? 0 : w.dtype == DT_Q8_0 ? 1 : w.dtype == DT_Q4_0 ? 2 : 3;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_done[dev][di]) {
        // the dynamic limit is the opt-in maximum minus the kernel's static shared memory
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaFuncAttributes fa = {};
        cudaError_t e = cudaFuncGetAttributes(&fa, k);
        if (e != cudaSuccess) return e;
        const size_t lim = (size_t)optin - fa.sharedSizeBytes;
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim);
        if (e != cudaSuccess) return e;
        attr_done[dev][di] = lim;
    }
    if (smem > attr_done[dev][di]) return cudaErrorInvalidConfiguration;
    // split partials through distributed shared memory when the splits fit in
    // one cluster and a partial ([npad][128] floats) fits in the drained rings
    const size_t rings = (ts ? (size_t)0 : (size_t)depth * ms * TC_M * 128) + (size_t)bdepth * npad * 128 +
                         (size_t)qdepth * ms * tc_stage_bytes(w.dtype);
    static const bool no_cluster = tc_knob("CMOLCU_TC_CLUSTER", 1) == 0;
    p.cluster = !no_cluster && ks > 1 && (size_t)npad * TC_M * 4 <= rings && tc_cluster_ok(k, ks, rb, smem) ? 1 : 0;
    cudaError_t e = launch_k(k_tc_xprep, dim3(npad), dim3(256), 0, st, pdl, a.x, a.x_ld, w.k, ncol, npad, a.norm_w,
                             a.eps, s.xs);
    if (e != cudaSuccess) return e;
    return tc_launch(k, dim3(rb, ks), smem, st, pdl, p.cluster ? ks : 1, p);
}
