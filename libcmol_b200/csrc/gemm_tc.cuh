// gemm_tc.cuh — the batched dequant matmul on the 5th-generation tensor
// cores (tcgen05), for decode steps that stack many sessions.
//
//   y(col, row) = sum_k deq(W[row, k]) * xn(col, k)       col < ncol <= 256
//
// The single-session GEMV (gemv.cuh) is exact f32 arithmetic on CUDA cores;
// once enough sessions share a step the product is a real dense
// contraction and this path takes over: weights are dequantised to f16 in
// shared memory, activations are rounded to f16, products accumulate in f32
// in tensor memory.  The rounding makes results differ from the CPU path by
// about 2^-11 relative per term (f16 mantissa), well inside the engine's
// logit tolerance.
//
// Two kernels:
//   k_tc_xprep : xn = x (or RMSNorm(x) * gains) -> f16, written in the
//                shared-memory image the MMA reads: per 64-value k-block,
//                npad rows of 128 bytes, 16-byte chunks XOR-swizzled by
//                (row % 8) (the K-major 128-byte-swizzle canonical layout)
//   k_tc_gemm  : CTA = 128 weight rows x a range of K-chunks.  Warp 0
//                bulk-copies the quantised K-chunk (K-chunk-major planes,
//                qweight.cuh) and the activation k-blocks; warps 2..9
//                dequantise k-block tiles of 128 x 64 into f16 (same
//                swizzled layout); warp 1 allocates tensor memory and one
//                thread issues tcgen05.mma (M=128, N=npad, K=16) per 16
//                values.  With one K range per row block the epilogue runs
//                straight from tensor memory; with several, each CTA writes
//                its partial sums and the last CTA of the row block adds
//                them in K order (deterministic) and runs the epilogue.
// Replaces the n > 1 use of kn->matmul (src/quant.c:334-566), whose n
// columns the reference re-dequantises per column.
#pragma once
#include "gemv.cuh"

#define TC_M 128
#define TC_KB 64
#define TC_MAX_N 256

struct TcScratch {
    uint16_t *xs;          // f16 activation image, >= k * npad halves
    float    *part;        // partial sums, >= part_floats
    size_t    part_floats;
    int      *counters;    // >= max row blocks, zero between launches
    int       max_row_blocks;
};

// True when the tensor-core path handles this weight format.
bool tc_supported(int dtype);

// Bytes of scratch the path needs for a [rows x k] weight at `ncol` columns.
void tc_scratch_need(int rows, int k, int ncol, size_t *xs_halves, size_t *part_floats, int *row_blocks);

// y = W . xn for `ncol` columns (x, y, norm and epilogue as in GemvArgs with
// x_inc = y_inc = 1).  Two launches (activation image, matmul).
cudaError_t tc_matmul(const GemvArgs &a, int ncol, int epi, const TcScratch &s, cudaStream_t st, bool pdl);
