// gemv.cuh — dequant-dot GEMV for one or two activation columns (sm_100a,
// CUDA cores fed by a bulk-copy pipeline).  Replaces the n=1 use of
// kn->matmul (src/quant.c:334-566 of the reference) on the decode path.
//
//   y(col,row) = sum_k deq(W[row,k]) * xn(col,k)        col < NCOL
//   xn = x                       when norm_w == NULL
//   xn = w[k] * (x[k] * inv_rms) otherwise (RMSNorm of src/model.c:90-97,
//                                fused into the prologue)
//
// Data movement.  A CTA owns one contiguous range of rows, walked in tiles
// of TR = CW*R rows (CW consumer warps, R rows each).  A tile moves in
// K-chunks of KC values (qweight.cuh: the whole row, or a multiple of 32
// payload chunks that keeps 32 rows near 24 KB).  One lane of the producer
// warp copies each (tile, K-chunk) into a shared-memory stage with one
// cp.async.bulk per plane — the rows of a K-chunk are contiguous in the
// K-chunk-major layout — and the stage's "full" mbarrier completes on the
// transaction byte count.  Weights do not depend on the previous kernel, so
// the producer never waits for it (programmatic dependent launch).  The
// consumer warps stage the activations, then each takes R rows of the tile:
// lane l owns 16-byte payload chunks l, l+32, ... of the K-chunk, loads a
// chunk's activations from shared memory once and reuses them for its R
// rows.  Consumers release a stage through its "empty" mbarrier.  Every wait
// is bounded (sync.cuh).  Two variants: CW = 8 (two CTAs an SM, ~100 KB of
// shared memory each: small decode matrices, so the next kernel streams
// while this one drains) and CW = 15 (one CTA an SM, up to ~216 KB: large
// matrices, more warps to issue the dequant arithmetic).
//
// Integer -> float without I2F.  A quantised value q (0..255 after biasing)
// placed in the low bits of a 32-bit word is the float q * 2^-149 (a
// subnormal).  The activations are stored pre-scaled by 2^85, so one fused
// multiply-add gives q * x * 2^-64 exactly (the product inside an fma is
// exact; FFMA keeps subnormals unless compiled with -ftz, which this build
// never is).  Per 16-value run the bias is removed with a precomputed run
// sum of the activations, and the per-block scale is applied once per run.
// The final row sum is scaled back by 2^64.  This costs about one PRMT and
// one FFMA per weight instead of a conversion, an add and an FFMA.
#pragma once
#include "common.cuh"
#include "qweight.cuh"
#include "sync.cuh"

enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

// Epilogue of the fused Q/K/V projection: global rows [0,D) are q,
// [D,D+KVD) k, [D+KVD,D+2KVD) v (global row = row_base + local row).  RoPE
// rotates q and k pairs with a host-built cos/sin table; k and v rows go
// straight into the session's KV page for position pos (src/attn.c:82-101).
struct EpiQKV {
    int          d_model, kv_dim, d_head, n_kv, page_tokens, layer, rope, row_base;
    const float2 *rope_cs;      // [pos][d_head/2] (cos, sin)
    const int   *pos;           // [ncol]; < 0 = inactive column
    const int   *slot;          // [ncol] session slot -> page-table row
    const int   *page_table;    // [slots][max_pages]
    int          max_pages;
    void        *kv_pages;      // this layer's region of the page pool (f32, or f16 when kv_f16)
    long long    page_elems;    // K/V values of one page in one layer: [K|V][kv head][token][d_head]
    int          n_pages;       // pages in the pool (bounds check)
    int          kv_f16;        // 1: values stored rounded to f16 (nearest, ties to even), chunks
                                //    swizzled by position (kv_swz)
};

// Stores the pair (v0, v1) at value index `off` of the KV pool.  off is even,
// so an f16 pair is one aligned 4-byte store.
__device__ __forceinline__ void kv_store_pair(const EpiQKV &e, long long off, float v0, float v1) {
    if (e.kv_f16) {
        *reinterpret_cast<__half2 *>(static_cast<__half *>(e.kv_pages) + off) = __floats2half2_rn(v0, v1);
    } else {
        float *p = static_cast<float *>(e.kv_pages) + off;
        p[0] = v0;
        p[1] = v1;
    }
}

// Stage geometry, computed on the host for one launch.
struct PipeCfg {
    int po[4];       // plane offsets inside a stage (TR rows of a full K-chunk each)
    int sb;          // stage bytes
    int nstage;      // pipeline depth
    int rows_per_cta;// contiguous rows per CTA (multiple of R)
    int cw;          // consumer warps (GEMV_CWARPS or GEMV_CWARPS_WIDE); a stage holds cw * R rows
};

struct GemvArgs {
    QWeight       w;
    const float  *x;  long long x_ld; int x_inc;     // x(col,i) = x[col*x_ld + i*x_inc]
    int           ncol;
    const float  *norm_w; float eps;
    float        *y;  long long y_ld; int y_inc;     // y(col,r) = y[col*y_ld + r*y_inc]
    EpiQKV        qkv;
    PipeCfg       pc;
    unsigned int *fault;                             // device fault word (may be NULL)
};

#define GEMV_CWARPS 8                          // consumer warps of the small-matrix variant
#define GEMV_THREADS ((GEMV_CWARPS + 1) * 32)  // + one producer warp
#define GEMV_CWARPS_WIDE 15                    // consumer warps of the large-matrix variant (16 warps in all: 128 registers a thread)
#define GEMV_MAX_STAGES 16

static constexpr float kXScale    = 38685626227668133590597632.0f;  // 2^85
static constexpr float kQScaleInv = 18446744073709551616.0f;        // 2^64

__device__ __forceinline__ float q_as_sub(uint32_t word, int byte) {
    return __uint_as_float(__byte_perm(word, 0u, 0x4440u | (uint32_t)byte));
}

// 16 FMAs of one run: four words of biased bytes against 16 activations.
__device__ __forceinline__ float dot_run16(const uint32_t w[4], const float4 *xr) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 xv = xr[i];
        acc = __fmaf_rn(q_as_sub(w[i], 0), xv.x, acc);
        acc = __fmaf_rn(q_as_sub(w[i], 1), xv.y, acc);
        acc = __fmaf_rn(q_as_sub(w[i], 2), xv.z, acc);
        acc = __fmaf_rn(q_as_sub(w[i], 3), xv.w, acc);
    }
    return acc;
}

// Spread the low 4 bits of v into bit 4 of each byte (the Q5_0 fifth bit).
__device__ __forceinline__ uint32_t spread4_bit4(uint32_t v) {
    return (v * 0x02040810u) & 0x10101010u;
}

// VPC: values per 16-byte payload chunk; CR: 16-value activation runs per chunk.
template <int DT> struct Fmt;
template <> struct Fmt<DT_Q8_0> { static constexpr int VPC = 16; static constexpr int CR = 1; };
template <> struct Fmt<DT_Q4_0> { static constexpr int VPC = 32; static constexpr int CR = 2; };
template <> struct Fmt<DT_Q5_0> { static constexpr int VPC = 32; static constexpr int CR = 2; };
template <> struct Fmt<DT_Q4_K> { static constexpr int VPC = 32; static constexpr int CR = 2; };
template <> struct Fmt<DT_Q6_K> { static constexpr int VPC = 32; static constexpr int CR = 2; };
template <> struct Fmt<DT_F16>  { static constexpr int VPC = 16; static constexpr int CR = 1; };
template <> struct Fmt<DT_F32>  { static constexpr int VPC = 16; static constexpr int CR = 1; };

// First activation index (within the row) of the two 16-value runs of chunk c.
template <int DT>
__device__ __forceinline__ void chunk_runs(int c, int &r0, int &r1) {
    if constexpr (DT == DT_Q8_0 || DT == DT_F16 || DT == DT_F32) {
        r0 = 16 * c; r1 = r0;
    } else if constexpr (DT == DT_Q4_0 || DT == DT_Q5_0) {
        r0 = 32 * c; r1 = r0 + 16;                       // low / high nibbles
    } else if constexpr (DT == DT_Q4_K) {
        int s = c >> 3, t = c & 7;                       // sub-blocks 2j, 2j+1
        r0 = 256 * s + 64 * (t >> 1) + 16 * (t & 1); r1 = r0 + 32;
    } else {                                             // Q6_K
        int s = c >> 3, t = c & 7;
        int glo = 4 * (t >> 2) + ((t & 3) >> 1);
        r0 = 256 * s + 32 * glo + 16 * (t & 1); r1 = r0 + 64;
    }
}

// Q4_K 6-bit scales and mins of the sub-block pair (2j, 2j+1) of a
// super-block, from its 12 packed bytes (src/quant.c:125-134) in three
// words w0 (bytes 0-3), w1 (4-7), w2 (8-11).  For j < 2 the pair is bytes
// 2j, 2j+1 of w0 (scales) and w1 (mins), low 6 bits; for j >= 2 the low
// 4 bits come from w2 (scales: low nibbles, mins: high nibbles) and the top
// 2 bits from bits 6-7 of the corresponding bytes of w0 / w1.  Both bytes
// of a pair are extracted at once; j is the same for every chunk a lane
// handles, so the selects below are loop invariant.
__device__ __forceinline__ void q4k_pair(uint32_t w0, uint32_t w1, uint32_t w2, int j, float &sc0, float &sc1,
                                         float &mn0, float &mn1) {
    const int h = (j & 1) * 16;
    const bool hi = j >= 2;
    const uint32_t mlo = hi ? 0x0F0Fu : 0x3F3Fu, mhi = hi ? 0x3030u : 0u;
    const uint32_t sp = (((hi ? w2 : w0) >> h) & mlo) | (((w0 >> h) >> 2) & mhi);
    const uint32_t mp = (((hi ? (w2 >> 4) : w1) >> h) & mlo) | (((w1 >> h) >> 2) & mhi);
    // small integers to float without a conversion instruction: 2^23 + v
    sc0 = __uint_as_float(0x4B000000u | (sp & 0xFFu)) - 8388608.0f;
    sc1 = __uint_as_float(0x4B000000u | ((sp >> 8) & 0xFFu)) - 8388608.0f;
    mn0 = __uint_as_float(0x4B000000u | (mp & 0xFFu)) - 8388608.0f;
    mn1 = __uint_as_float(0x4B000000u | ((mp >> 8) & 0xFFu)) - 8388608.0f;
}

// Contribution of local chunk cl (global chunk c) of stage row `tr`
// (2^-64 domain for quantised formats, the 2^85 domain for F16/F32).
// x0/x1: the chunk's two activation runs (scaled, 4 x float4 each),
// s0/s1: their run sums (2^-64 domain).
template <int DT>
__device__ __forceinline__ float chunk_math(const uint8_t *stage, const PipeCfg &pc, const int *st, int tr, int cl,
                                            int c, const float4 *x0, const float4 *x1, float s0, float s1) {
    const uint8_t *P0 = stage + pc.po[0] + tr * st[0];
    const uint8_t *P1 = stage + pc.po[1] + tr * st[1];
    if constexpr (DT == DT_Q8_0) {
        const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + cl * 16);
        float d = h2f(*reinterpret_cast<const uint16_t *>(P1 + (cl >> 1) * 2));
        uint32_t w[4] = {pl.x ^ 0x80808080u, pl.y ^ 0x80808080u, pl.z ^ 0x80808080u, pl.w ^ 0x80808080u};
        float acc = dot_run16(w, x0);
        return d * __fmaf_rn(-128.f, s0, acc);
    } else if constexpr (DT == DT_Q4_0 || DT == DT_Q5_0) {
        const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + cl * 16);
        float d = h2f(*reinterpret_cast<const uint16_t *>(P1 + cl * 2));
        uint32_t lo[4] = {pl.x & 0x0F0F0F0Fu, pl.y & 0x0F0F0F0Fu, pl.z & 0x0F0F0F0Fu, pl.w & 0x0F0F0F0Fu};
        uint32_t hi[4] = {(pl.x >> 4) & 0x0F0F0F0Fu, (pl.y >> 4) & 0x0F0F0F0Fu,
                          (pl.z >> 4) & 0x0F0F0F0Fu, (pl.w >> 4) & 0x0F0F0F0Fu};
        float bias = 8.f;
        if constexpr (DT == DT_Q5_0) {
            const uint32_t qh = *reinterpret_cast<const uint32_t *>(stage + pc.po[2] + tr * st[2] + cl * 4);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                lo[i] |= spread4_bit4((qh >> (4 * i)) & 15u);
                hi[i] |= spread4_bit4((qh >> (16 + 4 * i)) & 15u);
            }
            bias = 16.f;
        }
        float a0 = dot_run16(lo, x0);
        float a1 = dot_run16(hi, x1);
        return d * (__fmaf_rn(-bias, s0, a0) + __fmaf_rn(-bias, s1, a1));
    } else if constexpr (DT == DT_Q4_K) {
        const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + cl * 16);
        const uint4 h = *reinterpret_cast<const uint4 *>(P1 + (cl >> 3) * 16);
        float d    = h2f((uint16_t)(h.x & 0xFFFF));
        float dmin = h2f((uint16_t)(h.x >> 16));
        float sc0, sc1, mn0, mn1;
        q4k_pair(h.y, h.z, h.w, (c & 7) >> 1, sc0, sc1, mn0, mn1);
        uint32_t lo[4] = {pl.x & 0x0F0F0F0Fu, pl.y & 0x0F0F0F0Fu, pl.z & 0x0F0F0F0Fu, pl.w & 0x0F0F0F0Fu};
        uint32_t hi[4] = {(pl.x >> 4) & 0x0F0F0F0Fu, (pl.y >> 4) & 0x0F0F0F0Fu,
                          (pl.z >> 4) & 0x0F0F0F0Fu, (pl.w >> 4) & 0x0F0F0F0Fu};
        float a0 = dot_run16(lo, x0);
        float a1 = dot_run16(hi, x1);
        float db0 = d * sc0, mb0 = dmin * mn0;
        float db1 = d * sc1, mb1 = dmin * mn1;
        return __fmaf_rn(db0, a0, __fmaf_rn(-mb0, s0, __fmaf_rn(db1, a1, -mb1 * s1)));
    } else if constexpr (DT == DT_Q6_K) {
        const int t = c & 7, sbl = cl >> 3;
        const int glo = 4 * (t >> 2) + ((t & 3) >> 1);
        const uint4 pl = *reinterpret_cast<const uint4 *>(P0 + cl * 16);
        const uint4 qh = *reinterpret_cast<const uint4 *>(P1 + sbl * 64 + 32 * (t >> 2) + 16 * (t & 1));
        const int8_t *scp = reinterpret_cast<const int8_t *>(stage + pc.po[2] + tr * st[2] + sbl * 16 + 2 * glo + (t & 1));
        float d = h2f(*reinterpret_cast<const uint16_t *>(stage + pc.po[3] + tr * st[3] + sbl * 2));
        int sh = 2 * ((t & 3) >> 1);
        uint32_t pw[4] = {pl.x, pl.y, pl.z, pl.w};
        uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = (pw[i] & 0x0F0F0F0Fu) | (((hw[i] >> sh) & 0x03030303u) << 4);
            hi[i] = ((pw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (sh + 4)) & 0x03030303u) << 4);
        }
        float a0 = dot_run16(lo, x0);
        float a1 = dot_run16(hi, x1);
        float d0 = d * (float)scp[0], d1 = d * (float)scp[4];
        return __fmaf_rn(d0, __fmaf_rn(-32.f, s0, a0), d1 * __fmaf_rn(-32.f, s1, a1));
    } else if constexpr (DT == DT_F16) {
        const uint4 a = *reinterpret_cast<const uint4 *>(P0 + cl * 32);
        const uint4 b = *reinterpret_cast<const uint4 *>(P0 + cl * 32 + 16);
        uint32_t hw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const float *xf = reinterpret_cast<const float *>(x0);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hw[i]));
            acc = __fmaf_rn(f.x, xf[2 * i], acc);
            acc = __fmaf_rn(f.y, xf[2 * i + 1], acc);
        }
        return acc;
    } else {  // F32
        const float4 *w4 = reinterpret_cast<const float4 *>(P0 + cl * 64);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 w = w4[i];
            acc = __fmaf_rn(w.x, x0[i].x, acc);
            acc = __fmaf_rn(w.y, x0[i].y, acc);
            acc = __fmaf_rn(w.z, x0[i].z, acc);
            acc = __fmaf_rn(w.w, x0[i].w, acc);
        }
        return acc;
    }
}

template <int DT> __device__ __forceinline__ float final_scale() {
    if constexpr (DT == DT_F16 || DT == DT_F32) return 1.0f / kXScale;
    else return kQScaleInv;
}

// Rows 2i (gate) and 2i+1 (up) -> h[i] = silu(g) * u   (src/model.c:117-123)
__device__ __forceinline__ void epi_swiglu_pair(const GemvArgs &a, int row, int col, float g, float u) {
    float h = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    a.y[(long long)col * a.y_ld + (long long)(row / 2) * a.y_inc] = h;
}

// Operands the Q/K/V epilogue of rows (lrow, lrow+1) of column col reads
// from memory: the column's position, the page holding it (k/v rows) and the
// RoPE (cos, sin) of the pair (q/k rows).  They are fixed for the step, so a
// kernel can fetch them before its arithmetic.
struct QkvPre {
    int    pos, pg;
    float2 cs;
};

__device__ __forceinline__ QkvPre epi_qkv_fetch(const GemvArgs &a, int lrow, int col) {
    const EpiQKV &e = a.qkv;
    QkvPre q;
    q.pos = e.pos[col];
    q.pg = -1;
    q.cs = make_float2(1.f, 0.f);
    if (q.pos < 0) return q;
    const int row = e.row_base + lrow;
    const int D = e.d_model, KVD = e.kv_dim, hd = e.d_head;
    if (row >= D) {
        const int srow = e.slot ? e.slot[col] : col;
        q.pg = e.page_table[(long long)srow * e.max_pages + q.pos / e.page_tokens];
    }
    if (e.rope && row < D + KVD) q.cs = e.rope_cs[(long long)q.pos * (hd / 2) + ((row % hd) >> 1)];
    return q;
}

// Fused Q/K/V rows (lrow, lrow+1) of column col (local row numbering; the
// global row adds qkv.row_base): RoPE on q and k pairs, q to y, k and v into
// the column's KV page at its position.
__device__ __forceinline__ void epi_qkv_apply(const GemvArgs &a, int lrow, int col, float v0, float v1,
                                              const QkvPre &q) {
    const EpiQKV &e = a.qkv;
    const int row = e.row_base + lrow;
    const int pos = q.pos;
    if (pos < 0) return;
    const int D = e.d_model, KVD = e.kv_dim, hd = e.d_head;
    const bool is_v = row >= D + KVD;
    if (e.rope && !is_v) {
        // NORM-style pair rotation, src/model.c:137-166
        const float2 cs = q.cs;
        float n0 = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
        float n1 = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
        v0 = n0; v1 = n1;
    }
    if (row < D) {
        float *qo = a.y + (long long)col * a.y_ld;
        qo[row] = v0; qo[row + 1] = v1;
        return;
    }
    const int kvr = is_v ? row - D - KVD : row - D;
    const int head = kvr / hd, dim = kvr % hd;
    const int pg = q.pg;
    if (pg < 0 || pg >= e.n_pages) {   // never write outside the pool
        if (a.fault) atomicExch(a.fault, FAULT_BAD_PAGE);
        return;
    }
    const int t = pos % e.page_tokens;
    kv_store_pair(e, (long long)pg * e.page_elems +
                         (((long long)head * 2 + (is_v ? 1 : 0)) * e.page_tokens + t) * hd +
                         (e.kv_f16 ? kv_swz(pos, dim, hd) : dim),
                  v0, v1);
}

__device__ __forceinline__ void epi_qkv_pair(const GemvArgs &a, int lrow, int col, float v0, float v1) {
    epi_qkv_apply(a, lrow, col, v0, v1, epi_qkv_fetch(a, lrow, col));
}

// Epilogue operands prefetched for one warp's first row group: the old
// residual value (RESID) or the Q/K/V operands (QKV) of the lane's slot.
struct EpiPre {
    bool   valid;
    float  old;
    QkvPre q;
};

template <int NC, int R, int EPI>
__device__ __forceinline__ EpiPre gemv_epi_prefetch(const GemvArgs &a, int row0, int row_end, int lane) {
    EpiPre pre;
    pre.valid = false;
    pre.old = 0.f;
    pre.q.pos = -1;
    pre.q.pg = -1;
    pre.q.cs = make_float2(1.f, 0.f);
    if (row0 >= row_end) return pre;
    if constexpr (EPI == EPI_RESID) {
        if (lane < R * NC) {
            const int r = lane / NC, col = lane % NC, row = row0 + r;
            if (row < a.w.rows && col < a.ncol) pre.old = __ldcg(a.y + (long long)col * a.y_ld + (long long)row * a.y_inc);
        }
        pre.valid = true;
    } else if constexpr (EPI == EPI_QKV) {
        if (lane < (R / 2) * NC) {
            const int p = lane / NC, col = lane % NC;
            if (col < a.ncol && row0 + 2 * p + 1 < a.w.rows) pre.q = epi_qkv_fetch(a, row0 + 2 * p, col);
        }
        pre.valid = true;
    }
    return pre;
}

// Epilogue; vals[r*NC+col] hold the totals of rows row0..row0+R-1.
template <int NC, int R, int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs &a, int row0, const float *vals, int lane,
                                              const EpiPre *pre = nullptr) {
    const int rows = a.w.rows;
    if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
        if (lane < R * NC) {
            int r = lane / NC, col = lane % NC;
            int row = row0 + r;
            if (row < rows && col < a.ncol) {
                float *p = a.y + (long long)col * a.y_ld + (long long)row * a.y_inc;
                float v = vals[lane];
                if constexpr (EPI == EPI_RESID) *p = (pre && pre->valid ? pre->old : __ldcg(p)) + v;   // x += sublayer out (src/model.c:232,259)
                else *p = v;
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        if (lane < (R / 2) * NC) {
            int p = lane / NC, col = lane % NC;
            int row = row0 + 2 * p;
            if (row + 1 < rows && col < a.ncol)
                epi_swiglu_pair(a, row, col, vals[(2 * p) * NC + col], vals[(2 * p + 1) * NC + col]);
        }
    } else {  // EPI_QKV
        if (lane < (R / 2) * NC) {
            int p = lane / NC, col = lane % NC;
            if (row0 + 2 * p + 1 < rows && col < a.ncol) {
                if (pre && pre->valid)
                    epi_qkv_apply(a, row0 + 2 * p, col, vals[(2 * p) * NC + col], vals[(2 * p + 1) * NC + col], pre->q);
                else
                    epi_qkv_pair(a, row0 + 2 * p, col, vals[(2 * p) * NC + col], vals[(2 * p + 1) * NC + col]);
            }
        }
    }
}

// Dynamic shared memory.  Activations are stored lane-interleaved so that a
// warp reading "run p, float4 i" of 32 consecutive chunks touches 512
// contiguous bytes (no bank conflicts):
//   XS[col][c / 32][p][i][c % 32]  (float4)     RS[col][c / 32][p][c % 32]
// with c the chunk index (chunks padded to a multiple of 32).  Then the
// stages (128-byte aligned), then 2 * GEMV_MAX_STAGES mbarriers.
__host__ __device__ inline int gemv_chunks_padded(int k, int vpc) { return (k / vpc + 31) / 32 * 32; }
__host__ __device__ inline size_t gemv_x_bytes(int nc, int k, int vpc, int cr) {
    const size_t cp = (size_t)gemv_chunks_padded(k, vpc);
    return ((size_t)nc * cp * cr * (64 + 4) + 127) & ~(size_t)127;
}
__host__ __device__ inline size_t gemv_smem_total(int nc, int k, int vpc, int cr, const PipeCfg &pc) {
    return gemv_x_bytes(nc, k, vpc, cr) + (size_t)pc.nstage * pc.sb + 2 * GEMV_MAX_STAGES * 8;
}

template <int DT, int NC, int R, int EPI, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) k_gemv(GemvArgs a) {
    constexpr int VPC = Fmt<DT>::VPC;
    constexpr int CR = Fmt<DT>::CR;
    constexpr int TR = CW * R;
    const PipeCfg &pc = a.pc;
    const int K = a.w.k;
    const int C = K / VPC;
    const int CP = gemv_chunks_padded(K, VPC);
    float4 *XS = reinterpret_cast<float4 *>(cmolcu_smem);
    float *RS = reinterpret_cast<float *>(XS + (size_t)NC * CP * CR * 4);
    uint8_t *stages = cmolcu_smem + gemv_x_bytes(NC, K, VPC, CR);
    uint64_t *bar = reinterpret_cast<uint64_t *>(stages + (size_t)pc.nstage * pc.sb);
    uint64_t *full = bar, *empty = bar + GEMV_MAX_STAGES;
    __shared__ float red[CW][NC];
    __shared__ float inv_rms[NC];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        for (int s = 0; s < pc.nstage; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    // this CTA's contiguous row range, walked in stages of TR rows
    const int row_begin = min(a.w.rows, (int)blockIdx.x * pc.rows_per_cta);
    const int row_end = min(a.w.rows, row_begin + pc.rows_per_cta);
    const int ntile = (row_end - row_begin + TR - 1) / TR;
    const int nseq = ntile * a.w.nkc;

    if (warp == CW) {
        // ---------------- producer warp ----------------
        // one bulk copy per plane and stage: rows r0..r0+nrow of K-chunk j
        // are contiguous in the K-chunk-major layout (qweight.cuh)
        for (int seq = 0; seq < nseq; seq++) {
            const int s = seq % pc.nstage, n = seq / pc.nstage;
            const int r0 = row_begin + (seq / a.w.nkc) * TR;
            const int nrow = min(TR, row_end - r0);
            const int j = seq % a.w.nkc;
            if (n > 0 && !mbar_wait(&empty[s], (n - 1) & 1, a.fault, FAULT_GEMV_EMPTY)) return;
            if (lane == 0) {
                int bytes = 0;
#pragma unroll
                for (int p = 0; p < 4; p++)
                    if (p < a.w.nplanes) bytes += nrow * qw_stride(a.w, p, j);
                mbar_arrive_expect_tx(&full[s], (uint32_t)bytes);
                uint8_t *dst = stages + (size_t)s * pc.sb;
#pragma unroll
                for (int p = 0; p < 4; p++)
                    if (p < a.w.nplanes)
                        bulk_g2s(dst + pc.po[p], qw_row(a.w, p, j, r0), (uint32_t)(nrow * qw_stride(a.w, p, j)),
                                 &full[s]);
            }
            __syncwarp();
        }
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait();
    // the first tile's epilogue operands, in flight while the activations stage
    const EpiPre pre = gemv_epi_prefetch<NC, R, EPI>(a, row_begin + warp * R, row_end, lane);
    {
        // pass 1: RMS of each column (src/model.c:90-97), when normalising
        if (a.norm_w) {
            float ss[NC];
#pragma unroll
            for (int c = 0; c < NC; c++) ss[c] = 0.f;
            for (int i = tid; i < K; i += CW * 32) {
#pragma unroll
                for (int c = 0; c < NC; c++) {
                    float v = c < a.ncol ? a.x[(long long)c * a.x_ld + (long long)i * a.x_inc] : 0.f;
                    ss[c] = __fmaf_rn(v, v, ss[c]);
                }
            }
#pragma unroll
            for (int c = 0; c < NC; c++) {
                float v = warp_sum(ss[c]);
                if (lane == 0) red[warp][c] = v;
            }
            named_bar_sync(1, CW * 32);
            if (tid < NC) {
                float t = 0.f;
                for (int w = 0; w < CW; w++) t += red[w][tid];
                inv_rms[tid] = 1.0f / sqrtf(t / (float)K + a.eps);
            }
            named_bar_sync(1, CW * 32);
        }
        // pass 2: one thread per (column, chunk, run): normalise, scale by
        // 2^85, store interleaved, and store the run sum (2^-64 domain)
        for (int j = tid; j < NC * C * CR; j += CW * 32) {
            const int col = j / (C * CR), rem = j % (C * CR), c = rem / CR, p = rem % CR;
            int q0, q1;
            chunk_runs<DT>(c, q0, q1);
            const int r = p ? q1 : q0;
            float v[16];
            const float *src = a.x + (long long)col * a.x_ld + (long long)r * a.x_inc;
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = col < a.ncol ? src[(long long)i * a.x_inc] : 0.f;
            if (a.norm_w) {
                const float ir = inv_rms[col];
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = __fmul_rn(a.norm_w[r + i], __fmul_rn(v[i], ir));
            }
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) { v[i] *= kXScale; t += v[i]; }
            float4 *dst = XS + ((size_t)col * CP * CR * 4 + (size_t)(c >> 5) * CR * 32 * 4 + (size_t)p * 4 * 32) + (c & 31);
#pragma unroll
            for (int i = 0; i < 4; i++) dst[i * 32] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            RS[(size_t)col * CP * CR + (size_t)(c >> 5) * CR * 32 + p * 32 + (c & 31)] = t * __int_as_float(1);
        }
        named_bar_sync(1, CW * 32);
    }

    int seq = 0;
    for (int ti = 0; ti < ntile; ti++) {
        const int row0 = row_begin + ti * TR + warp * R;
        float acc[R * NC];
#pragma unroll
        for (int i = 0; i < R * NC; i++) acc[i] = 0.f;
        for (int kci = 0; kci < a.w.nkc; kci++, seq++) {
            const int s = seq % pc.nstage, n = seq / pc.nstage;
            if (!mbar_wait(&full[s], n & 1, a.fault, FAULT_GEMV_FULL)) return;
            const uint8_t *stage = stages + (size_t)s * pc.sb;
            const int CC = qw_chunk_values(a.w, kci) / VPC;
            const int c0 = kci * (a.w.kc / VPC);
            int st[4];
#pragma unroll
            for (int p = 0; p < 4; p++) st[p] = qw_stride(a.w, p, kci);
            if (row0 < row_end) {
                for (int cl = lane; cl < CC; cl += 32) {
                    const int c = c0 + cl;
#pragma unroll
                    for (int col = 0; col < NC; col++) {
                        const float4 *xb = XS + (size_t)col * CP * CR * 4 + (size_t)(c >> 5) * CR * 32 * 4 + (c & 31);
                        const float *rb = RS + (size_t)col * CP * CR + (size_t)(c >> 5) * CR * 32 + (c & 31);
                        float4 x0[4], x1[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) x0[i] = xb[i * 32];
                        const float s0 = rb[0];
                        float s1 = s0;
                        if constexpr (CR == 2) {
#pragma unroll
                            for (int i = 0; i < 4; i++) x1[i] = xb[(4 + i) * 32];
                            s1 = rb[32];
                        } else {
#pragma unroll
                            for (int i = 0; i < 4; i++) x1[i] = x0[i];
                        }
#pragma unroll
                        for (int r = 0; r < R; r++)
                            acc[r * NC + col] += chunk_math<DT>(stage, pc, st, warp * R + r, cl, c, x0, x1, s0, s1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (row0 < row_end) {
            float vals[R * NC];
#pragma unroll
            for (int i = 0; i < R * NC; i++) vals[i] = warp_sum(acc[i]) * final_scale<DT>();
            gemv_epilogue<NC, R, EPI>(a, row0, vals, lane, ti == 0 ? &pre : nullptr);
        }
    }
}
