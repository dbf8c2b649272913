// gemm_tc.cu — batched dequant matmul on tcgen05 tensor cores (see gemm_tc.cuh).
#include "gemm_tc.cuh"
#include "gemv_launch.cuh"

#include <algorithm>

#define TC_DQW 8                          // dequantising warps (2..9)
#define TC_THREADS ((2 + TC_DQW) * 32)    // + producer warp 0, MMA warp 1
#define TC_DQT (TC_DQW * 32)
#define TC_MAX_DEPTH 8

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

// 16-byte asynchronous copy global -> shared through the load/store unit,
// and the arrival of this thread on `bar` once its earlier copies landed
// (the mbarrier counts one arrival per issuing thread).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
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
    for (int c = tid; c < K / 8; c += 256) {
        const int k0 = c * 8, kb = k0 >> 6, ch = (k0 & 63) >> 3;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float t = live ? xc[k0 + i] : 0.f;
            if (live && norm_w) t = __fmul_rn(norm_w[k0 + i], __fmul_rn(t, ir));
            v[i] = t;
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
    GemvArgs        g;                 // weight, y, epilogue fields
    int             epi, ncol, npad;
    const uint16_t *xs;
    int             nslice;            // K-slices of the matrix (slices never cross a K-chunk)
    int             ksplit, slices_per_split;
    float          *part;
    int            *counters;
    uint32_t        tmem_cols;
    int             depth;             // A / B tile ring depth (<= TC_MAX_DEPTH)
    int             qdepth;            // quantised-stage ring depth (<= TC_MAX_QD)
};

// Row stride, in a quantised stage, of plane p of format DT for one 256-value
// slice: the slice's bytes rounded to 16, then to an odd multiple of 16 so
// that the 8 lanes of a shared-memory phase reading 8 consecutive rows hit 8
// different 16-byte bank groups.
__host__ __device__ constexpr int tc_sp(int dt, int p) {
    const int b = dt == DT_Q8_0 ? (p == 0 ? 256 : p == 1 ? 16 : 0)
                : dt == DT_Q5_0 ? (p == 0 ? 128 : p == 1 ? 16 : p == 2 ? 32 : 0)
                : (p == 0 ? 128 : p == 1 ? 16 : 0);          // Q4_0, Q4_K
    return b == 0 ? 0 : ((b / 16) % 2 == 0 ? b + 16 : b);
}
__host__ __device__ constexpr int tc_stage_bytes(int dt) {
    return TC_M * (tc_sp(dt, 0) + tc_sp(dt, 1) + tc_sp(dt, 2));
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

// 16 dequantised values of row r, values [v, v + 16) of the K-chunk held in
// the quantised stage (GGUF block arithmetic of src/quant.c:152-194), as 8
// packed f16 pairs.  No conversion instructions: a small unsigned integer u
// becomes the f16 1024 + u by placing it under the exponent bits 0x6400
// (one byte permute per pair), and the f32 2^23 + u under 0x4B000000.
//   Q8_0, Q4_0, Q5_0: q is exact in f16 and the block scale d is an f16, so
//                     d * q in f16 arithmetic is the f16 rounding of the exact
//                     value (the same as rounding the f32 product).
//   Q4_K:             d * sc * q - dmin * mn in f32 (sc, mn 6-bit), then f16.
__device__ __forceinline__ uint32_t h2_from_bytes(uint32_t w, uint32_t sel) {
    // bytes of w selected by sel into the low byte of each half, 0x64 above
    return __byte_perm(w, 0x64646464u, sel);
}

template <int DT>
__device__ __forceinline__ void tc_dequant16(const uint8_t *P0, const uint8_t *P1, const uint8_t *P2, int v,
                                             uint32_t out[8]) {
    if constexpr (DT == DT_Q4_K) {
        // one super-block per slice: v in [0, 256)
        const int pj = v >> 6, half = (v >> 5) & 1, sub = (v >> 4) & 1;
        const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + 32 * pj + 16 * sub);
        const uint4 h = *reinterpret_cast<const uint4 *>(P1);
        const float d = h2f((uint16_t)(h.x & 0xFFFF)), dmin = h2f((uint16_t)(h.x >> 16));
        float sc0, sc1, mn0, mn1;
        q4k_pair(h.y, h.z, h.w, pj, sc0, sc1, mn0, mn1);
        const float a = d * (half ? sc1 : sc0), m = dmin * (half ? mn1 : mn0);
        const uint32_t w[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t t = half ? ((w[i] >> 4) & 0x0F0F0F0Fu) : (w[i] & 0x0F0F0F0Fu);
            float f[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                f[j] = __fmaf_rn(a, __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7540u | j)) - 8388608.0f, -m);
            out[2 * i] = pack_h2(f[0], f[1]);
            out[2 * i + 1] = pack_h2(f[2], f[3]);
        }
    } else {
        const int b = v >> 5, hh = (v >> 4) & 1;
        uint32_t w[4];
        __half bias;
        __half d;
        if constexpr (DT == DT_Q8_0) {
            const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + b * 32 + 16 * hh);
            d = __ushort_as_half(*reinterpret_cast<const uint16_t *>(P1 + b * 2));
            w[0] = pl.x ^ 0x80808080u; w[1] = pl.y ^ 0x80808080u;      // int8 -> unsigned + 128
            w[2] = pl.z ^ 0x80808080u; w[3] = pl.w ^ 0x80808080u;
            bias = __ushort_as_half((uint16_t)0x6480);                  // 1024 + 128
        } else {
            const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + b * 16);
            d = __ushort_as_half(*reinterpret_cast<const uint16_t *>(P1 + b * 2));
            const uint32_t raw[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
            for (int i = 0; i < 4; i++) w[i] = hh ? ((raw[i] >> 4) & 0x0F0F0F0Fu) : (raw[i] & 0x0F0F0F0Fu);
            if constexpr (DT == DT_Q5_0) {
                const uint32_t qh = *reinterpret_cast<const uint32_t *>(P2 + b * 4);
#pragma unroll
                for (int i = 0; i < 4; i++) w[i] |= spread4_bit4((qh >> (16 * hh + 4 * i)) & 15u);
                bias = __ushort_as_half((uint16_t)0x6410);              // 1024 + 16
            } else {
                bias = __ushort_as_half((uint16_t)0x6408);              // 1024 + 8
            }
        }
        const __half2 b2 = __halves2half2(bias, bias), d2 = __halves2half2(d, d);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = h2_from_bytes(w[i], 0x5140u), hi = h2_from_bytes(w[i], 0x5342u);
            __half2 x0 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&lo), b2), d2);
            __half2 x1 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&hi), b2), d2);
            out[2 * i] = *reinterpret_cast<const uint32_t *>(&x0);
            out[2 * i + 1] = *reinterpret_cast<const uint32_t *>(&x1);
        }
    }
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

template <int DT>
__global__ void __launch_bounds__(TC_THREADS, 2) k_tc_gemm(const __grid_constant__ TcParams p) {
    const QWeight &w = p.g.w;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = blockIdx.x, ks = blockIdx.y;
    const int m0 = rb * TC_M;
    const int npad = p.npad;
    const int s0 = ks * p.slices_per_split, s1 = min(p.nslice, s0 + p.slices_per_split);
    constexpr int SP0 = tc_sp(DT, 0), SP1 = tc_sp(DT, 1), SP2 = tc_sp(DT, 2);
    constexpr int QOFF1 = TC_M * SP0, QOFF2 = TC_M * (SP0 + SP1), QB = tc_stage_bytes(DT);

    // shared memory: A tiles, B tiles (1024-aligned), quantised stages, barriers
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)cmolcu_smem + 1023) & ~(uintptr_t)1023);
    const int D = p.depth, QD = p.qdepth;
    uint8_t *A = base;                                        // D x 16 KB
    uint8_t *B = A + (size_t)D * TC_M * 128;                  // D x npad * 128
    uint8_t *Q = B + (size_t)D * npad * 128;                  // QD x QB
    uint64_t *bars = reinterpret_cast<uint64_t *>(Q + (size_t)QD * QB);
    uint64_t *accfull = bars, *qfull = bars + 1, *qempty = qfull + TC_MAX_QD, *afull = qempty + TC_MAX_QD,
             *aempty = afull + TC_MAX_DEPTH, *bfull = aempty + TC_MAX_DEPTH, *bempty = bfull + TC_MAX_DEPTH;
    __shared__ uint32_t s_tmem;
    __shared__ int s_last;

    if (tid == 0) {
        for (int i = 0; i < QD; i++) {
            mbar_init(&qfull[i], 32);       // one cp.async arrival per producer lane
            mbar_init(&qempty[i], TC_DQW);
        }
        for (int i = 0; i < D; i++) {
            mbar_init(&afull[i], TC_DQW);
            mbar_init(&aempty[i], 1);
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        mbar_init(accfull, 1);
        fence_mbar_init();
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
        // ---------------- producer: quantised slices (all lanes) and activation blocks (lane 0) --------
        const int nrow = min(TC_M, w.prow - m0);
        int bn = 0;
        bool ok = true;
        for (int t = s0; t < s1 && ok; t++) {
            const int li = t - s0, stg = li % QD, use = li / QD;
            if (use > 0 && !mbar_wait(&qempty[stg], (use - 1) & 1, p.g.fault, FAULT_GEMV_EMPTY)) { ok = false; break; }
            int j, off, len;
            tc_slice(w, t, j, off, len);
            // 16-byte chunks of every row of every plane (consecutive lanes take
            // consecutive chunks of a row: coalesced reads of the K-chunk-major planes)
            const int c0 = round16(qw_plane_bytes(DT, 0, len)) / 16;
            const int c1 = round16(qw_plane_bytes(DT, 1, len)) / 16;
            const int c2 = DT == DT_Q5_0 ? round16(qw_plane_bytes(DT, 2, len)) / 16 : 0;
            const int o0 = qw_plane_bytes(DT, 0, off), o1 = qw_plane_bytes(DT, 1, off), o2 = qw_plane_bytes(DT, 2, off);
            uint8_t *q = Q + (size_t)stg * QB;
            for (int idx = lane; idx < nrow * c0; idx += 32) {
                const int r = idx / c0, c = idx % c0;
                cp_async16(q + r * SP0 + 16 * c, qw_row(w, 0, j, m0 + r) + o0 + 16 * c);
            }
            for (int idx = lane; idx < nrow * c1; idx += 32) {
                const int r = idx / c1, c = idx % c1;
                cp_async16(q + QOFF1 + r * SP1 + 16 * c, qw_row(w, 1, j, m0 + r) + o1 + 16 * c);
            }
            if constexpr (DT == DT_Q5_0) {
                for (int idx = lane; idx < nrow * c2; idx += 32) {
                    const int r = idx / c2, c = idx % c2;
                    cp_async16(q + QOFF2 + r * SP2 + 16 * c, qw_row(w, 2, j, m0 + r) + o2 + 16 * c);
                }
            }
            cp_async_arrive(&qfull[stg]);
            if (lane == 0) {
                if (li == 0) pdl_wait();   // the activation image comes from the previous kernel
                const int g0 = (j * w.kc + off) / TC_KB;
                for (int i = 0; i < len / TC_KB; i++, bn++) {
                    const int slot = bn % D, u = bn / D;
                    if (u > 0 && !mbar_wait(&bempty[slot], (u - 1) & 1, p.g.fault, FAULT_GEMV_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&bfull[slot], (uint32_t)(npad * 128));
                    bulk_g2s(B + (size_t)slot * npad * 128, p.xs + (size_t)(g0 + i) * npad * 64, (uint32_t)(npad * 128),
                             &bfull[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t)(npad >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
            for (int i = 0; i < nkb; i++) {
                const int slot = i % D, use = i / D;
                mbar_wait(&afull[slot], use & 1, p.g.fault, FAULT_GEMV_FULL);
                mbar_wait(&bfull[slot], use & 1, p.g.fault, FAULT_GEMV_FULL);
                tc_fence_after();
                const uint32_t a_addr = smem_u32(A + slot * TC_M * 128), b_addr = smem_u32(B + (size_t)slot * npad * 128);
#pragma unroll
                for (int k = 0; k < TC_KB / 16; k++)
                    tc_mma(tmem, tc_desc(a_addr + 32 * k), tc_desc(b_addr + 32 * k), idesc, (i | k) != 0);
                tc_commit(&aempty[slot]);
                tc_commit(&bempty[slot]);
            }
            tc_commit(accfull);
        }
    } else {
        // ---------------- dequantise ----------------
        const int dt = tid - 64;
        int i = 0;
        for (int t = s0; t < s1; t++) {
            const int li = t - s0, stg = li % QD;
            mbar_wait(&qfull[stg], (li / QD) & 1, p.g.fault, FAULT_GEMV_FULL);
            int j, off, len;
            tc_slice(w, t, j, off, len);
            const uint8_t *q = Q + (size_t)stg * QB;
            for (int ib = 0; ib < len / TC_KB; ib++, i++) {
                const int slot = i % D, use = i / D;
                if (use > 0) mbar_wait(&aempty[slot], (use - 1) & 1, p.g.fault, FAULT_GEMV_EMPTY);
                uint8_t *tile = A + slot * TC_M * 128;
                // task = (row r, 16-value run qq): 128 rows x 4 runs
#pragma unroll
                for (int tt = 0; tt < (TC_M * 4) / TC_DQT; tt++) {
                    const int task = dt + TC_DQT * tt, r = task >> 2, qq = task & 3;
                    uint32_t h[8];
                    tc_dequant16<DT>(q + r * SP0, q + QOFF1 + r * SP1, q + QOFF2 + r * SP2, ib * TC_KB + 16 * qq, h);
                    uint4 *row = reinterpret_cast<uint4 *>(tile + r * 128);
                    row[(2 * qq) ^ (r & 7)] = make_uint4(h[0], h[1], h[2], h[3]);
                    row[(2 * qq + 1) ^ (r & 7)] = make_uint4(h[4], h[5], h[6], h[7]);
                }
                fence_proxy_async_smem();   // the tensor core reads the tile through the async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[slot]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&qempty[stg]);
        }
        // ---------------- epilogue: tensor memory -> registers ----------------
        if (warp < 6) {
            const int quarter = warp & 3;                 // the TMEM lanes this warp may read
            const int row = m0 + 32 * quarter + lane;
            mbar_wait(accfull, 0, p.g.fault, FAULT_GEMV_FULL);
            tc_fence_after();
            if (p.ksplit == 1) pdl_wait();
            for (int c0 = 0; c0 < npad; c0 += 16) {
                float v[16];
                tc_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, v);
                if (p.ksplit == 1) {
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 1);
                        tc_epilogue(p, row, c0 + e, v[e], partner);
                    }
                } else {
                    float *pp = p.part + ((size_t)(rb * p.ksplit + ks) * npad + c0) * TC_M + (row - m0);
#pragma unroll
                    for (int e = 0; e < 16; e++) pp[(size_t)e * TC_M] = v[e];
                }
            }
        }
    }

    // ---------------- split-K: the last CTA of the row block adds the partials ----------------
    tc_fence_before();
    __syncthreads();
    if (p.ksplit > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&p.counters[rb], 1) == p.ksplit - 1;
        __syncthreads();
        if (s_last) {
            __threadfence();
            pdl_wait();
            // thread = (row pair, column): the even row's thread applies pair epilogues
            for (int idx = tid; idx < (TC_M / 2) * npad; idx += TC_THREADS) {
                const int rp = idx % (TC_M / 2), col = idx / (TC_M / 2);
                const int r = 2 * rp;
                float v0 = 0.f, v1 = 0.f;
                for (int s = 0; s < p.ksplit; s++) {
                    const float *pp = p.part + ((size_t)(rb * p.ksplit + s) * npad + col) * TC_M + r;
                    v0 += __ldcg(pp);
                    v1 += __ldcg(pp + 1);
                }
                const int row = m0 + r;
                if (p.epi == EPI_STORE || p.epi == EPI_RESID) {
                    tc_epilogue(p, row, col, v0, v1);
                    tc_epilogue(p, row + 1, col, v1, v0);
                } else {
                    tc_epilogue(p, row, col, v0, v1);
                }
            }
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
static void tc_rings(int dt, int npad, int &depth, int &qdepth, size_t &smem, int &per_sm) {
    const size_t qb = (size_t)tc_stage_bytes(dt), bars = (1 + 2 * TC_MAX_QD + 4 * TC_MAX_DEPTH) * 8;
    const size_t per_slot = (size_t)TC_M * 128 + (size_t)npad * 128;
    for (per_sm = 2; per_sm >= 1; per_sm--) {
        const long long budget = per_sm == 2 ? 112LL * 1024 : 220LL * 1024;
        qdepth = per_sm == 2 ? 2 : 3;
        const long long room = budget - 1024 - (long long)(qdepth * qb) - (long long)bars;
        depth = (int)std::min<long long>(TC_MAX_DEPTH, room / (long long)per_slot);
        smem = 1024 + (size_t)std::max(depth, 2) * per_slot + (size_t)qdepth * qb + bars;
        if (depth >= 2 && (long long)smem <= budget) return;
    }
    per_sm = 1;
    depth = 2;
    qdepth = 2;
    smem = 1024 + 2 * per_slot + 2 * qb + bars;
}

static int tc_nslice(int k, int kc) {
    const int nkc = (k + kc - 1) / kc;
    const int last = k - (nkc - 1) * kc;
    return (nkc - 1) * (kc / TC_SV) + (last + TC_SV - 1) / TC_SV;
}

static void tc_split(int rows, int nslice, int per_sm, int &rblocks, int &ksplit, int &sps) {
    const int slots = device_sm_count() * per_sm;
    rblocks = (rows + TC_M - 1) / TC_M;
    ksplit = std::max(1, std::min(nslice, slots / rblocks));    // one wave
    sps = (nslice + ksplit - 1) / ksplit;
    ksplit = (nslice + sps - 1) / sps;
}

void tc_scratch_need(int rows, int k, int ncol, size_t *xs_halves, size_t *part_floats, int *row_blocks) {
    const int npad = tc_npad(ncol);
    *xs_halves = (size_t)k * npad;
    int rb, ks, sps;
    tc_split(rows, k / TC_KB, 2, rb, ks, sps);     // an upper bound on the split of any format
    *part_floats = ks > 1 ? (size_t)rb * ks * npad * TC_M : 0;
    *row_blocks = rb;
}

typedef void (*tc_kernel_t)(TcParams);

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
    int depth, qdepth, per_sm;
    size_t smem;
    tc_rings(w.dtype, npad, depth, qdepth, smem, per_sm);
    const int nslice = tc_nslice(w.k, w.kc);
    int rb, ks, sps;
    tc_split(w.rows, nslice, per_sm, rb, ks, sps);
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
    p.tmem_cols = npad <= 32 ? 32 : npad <= 64 ? 64 : npad <= 128 ? 128 : 256;
    p.depth = depth;
    p.qdepth = qdepth;
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
    cudaError_t e = launch_k(k_tc_xprep, dim3(npad), dim3(256), 0, st, pdl, a.x, a.x_ld, w.k, ncol, npad, a.norm_w,
                             a.eps, s.xs);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(rb, ks), dim3(TC_THREADS), smem, st, pdl, p);
}
