// qweight.cuh — device layout of a quantised weight matrix.
//
// GGUF stores a row as an array of packed blocks (src/quant.c:78-105 of the
// reference); Q8_0 (34 B), Q5_0 (22 B), Q4_0 (18 B) and Q6_K (210 B) blocks
// break 16-byte alignment.  At upload the matrix is cut into K-chunks of kc
// values (kc a multiple of the block size; one chunk when the row is short)
// and every block is split into planes.  A plane of a K-chunk is stored row
// major with its rows padded to 16 bytes, and the row count is padded to 32:
//
//   plane p, K-chunk j, row r  at  p[p] + j * prow * cs[p] + r * stride(p, j)
//   stride(p, j) = cs[p] for full chunks, cl[p] for the last (shorter) one
//
// so ANY contiguous range of rows of one K-chunk of one plane is a single
// 16-byte aligned block that one bulk copy moves.  The bytes are the GGUF
// bytes, re-laid out; one pass streams the tensor's GGUF size plus the
// padding of short scale rows.
//
//   dtype  payload plane (q)         plane a                 plane b          plane c
//   Q8_0   int8 qs       [kc]        f16 d [kc/32]           -                -
//   Q4_0   nibbles       [kc/2]      f16 d [kc/32]           -                -
//   Q5_0   nibbles       [kc/2]      f16 d [kc/32]           u32 qh [kc/32]   -
//   Q4_K   nibbles       [kc/2]      16 B header [kc/256]    -                -
//          (header = f16 d, f16 dmin, 12 B packed 6-bit scales/mins)
//   Q6_K   ql            [kc/2]      qh [kc/4]               i8 sc [kc/16]    f16 d [kc/256]
//   F16    half          [kc]        -                       -                -
//   F32    float         [kc]        -                       -                -
//
// Within a plane the GGUF byte order of each block is kept, so nibble j of
// a Q4_0/Q5_0 block still holds value j (low) and j+16 (high), and the Q4_K /
// Q6_K sub-block interleaving is that of src/quant.c:172-232.
#pragma once
#include "common.cuh"

#define QW_ROW_PAD 32

struct QWeight {
    int      dtype;
    int      rows;       // real rows (allocation holds rows rounded up to 32)
    int      prow;       // padded rows
    int      k;
    int      kc;         // values per K-chunk
    int      nkc;        // K-chunks
    int      nplanes;
    uint8_t *p[4];       // planes: q, a, b, c
    int      cs[4];      // row stride (bytes) of a full K-chunk of each plane
    int      cl[4];      // row stride of the last K-chunk
    size_t   bytes;      // GGUF bytes of the tensor
};

// Unpadded bytes of `kv` values of one row in plane `pl`.
__host__ __device__ inline int qw_plane_bytes(int dt, int pl, int kv) {
    switch (dt) {
    case DT_Q8_0: return pl == 0 ? kv : pl == 1 ? kv / 16 : 0;
    case DT_Q4_0: return pl == 0 ? kv / 2 : pl == 1 ? kv / 16 : 0;
    case DT_Q5_0: return pl == 0 ? kv / 2 : pl == 1 ? kv / 16 : pl == 2 ? kv / 8 : 0;
    case DT_Q4_K: return pl == 0 ? kv / 2 : pl == 1 ? kv / 16 : 0;
    case DT_Q6_K: return pl == 0 ? kv / 2 : pl == 1 ? kv / 4 : pl == 2 ? kv / 16 : pl == 3 ? kv / 128 : 0;
    case DT_F16: return pl == 0 ? kv * 2 : 0;
    case DT_F32: return pl == 0 ? kv * 4 : 0;
    default: return 0;
    }
}

__host__ __device__ inline int qw_nplanes(int dt) {
    switch (dt) {
    case DT_Q8_0: case DT_Q4_0: case DT_Q4_K: return 2;
    case DT_Q5_0: return 3;
    case DT_Q6_K: return 4;
    case DT_F16: case DT_F32: return 1;
    default: return 0;
    }
}

__host__ __device__ inline int round16(int b) { return (b + 15) & ~15; }

// Values in K-chunk j.
__host__ __device__ inline int qw_chunk_values(const QWeight &w, int j) {
    return j < w.nkc - 1 ? w.kc : w.k - (w.nkc - 1) * w.kc;
}

__host__ __device__ inline int qw_stride(const QWeight &w, int p, int j) {
    return j < w.nkc - 1 ? w.cs[p] : w.cl[p];
}

// Address of row r of K-chunk j in plane p.
__host__ __device__ inline uint8_t *qw_row(const QWeight &w, int p, int j, long long r) {
    return w.p[p] + (long long)j * w.prow * w.cs[p] + r * qw_stride(w, p, j);
}

// Default K-chunk: the whole row when 32 rows of it stay near 24 KB,
// otherwise the largest multiple of 32 payload chunks (512 values for the
// 16-value-chunk formats Q8_0/F16/F32, 1024 for the others) that does, so
// every lane of a warp walking a K-chunk has work; the largest multiple of
// the block size when not even one such unit fits.
__host__ inline int qw_default_kc(int dt, int k) {
    const int bv = dt_block_values(dt);
    int per32 = 0;
    for (int p = 0; p < qw_nplanes(dt); p++) per32 += round16(qw_plane_bytes(dt, p, k));
    if (32 * per32 <= 24 * 1024 || bv <= 0) return k;
    const int unit = (dt == DT_Q8_0 || dt == DT_F16 || dt == DT_F32) ? 512 : 1024;
    auto fits = [&](int kc) {
        int b = 0;
        for (int p = 0; p < qw_nplanes(dt); p++) b += round16(qw_plane_bytes(dt, p, kc));
        return 32 * b <= 24 * 1024;
    };
    if (unit % bv == 0 && fits(unit)) {
        int kc = unit;
        while (kc + unit < k && fits(kc + unit)) kc += unit;
        return kc;
    }
    // bytes per value (all planes) ~ per32 / k
    long long kc = (long long)24 * 1024 * k / (32LL * per32);
    kc = kc / bv * bv;
    if (kc < bv) kc = bv;
    if (kc >= k) return k;
    return (int)kc;
}

// Total bytes of the padded planes; fills the geometry of `w` (p[] = offsets).
__host__ inline size_t qw_layout(QWeight &w, int dt, int rows, int k, int kc) {
    w.dtype = dt;
    w.rows = rows;
    w.prow = (rows + QW_ROW_PAD - 1) / QW_ROW_PAD * QW_ROW_PAD;
    w.k = k;
    w.kc = kc;
    w.nkc = (k + kc - 1) / kc;
    w.nplanes = qw_nplanes(dt);
    size_t tot = 0;
    for (int p = 0; p < 4; p++) {
        if (p < w.nplanes) {
            w.cs[p] = round16(qw_plane_bytes(dt, p, kc));
            w.cl[p] = round16(qw_plane_bytes(dt, p, k - (w.nkc - 1) * kc));
            size_t sz = (size_t)w.prow * ((size_t)(w.nkc - 1) * w.cs[p] + w.cl[p]);
            w.p[p] = (uint8_t *)(uintptr_t)tot;   // offset, rebased by the caller
            tot += (sz + 255) & ~(size_t)255;
        } else {
            w.cs[p] = w.cl[p] = 0;
            w.p[p] = nullptr;
        }
    }
    w.bytes = (size_t)rows * dt_row_bytes(k, dt);
    return tot;
}

// Largest k the GEMV stages in shared memory per column (floats).
#define CMOLCU_GEMV_MAX_K 16384
