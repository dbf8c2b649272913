// attention.cuh — GQA decode attention over the paged KV cache.
//
// Replaces step 5 of cmol_attn_forward (src/attn.c:103-137 of the reference):
// for every query head h of a session at position pos,
//   out_h = sum_{t<=pos} softmax_t(q_h . k_t / sqrt(d_head)) v_t
// with k/v of kv head h * n_kv / n_heads.  The context is split into chunks
// of `split_tokens` (flash-decoding): CTA (split s, kv head, column) copies
// the K and V blocks of its chunk's pages into shared memory with bulk
// copies (once for all query heads of the group), scores every token of the
// chunk, and writes a partial (max, sum, acc[d_head]) per head.  The last CTA
// of a (column, kv head) to finish — found with an atomic counter — merges
// the partials in split order (deterministic) and resets the counter.
#pragma once
#include "common.cuh"

struct AttnArgs {
    const float *q;          // [ncol][q_ld] query rows (RoPE applied)
    long long    q_ld;
    float       *out;        // [ncol][out_ld]
    long long    out_ld;
    const int   *pos;        // [ncol]; < 0 = inactive column
    const int   *slot;       // [ncol] -> page-table row
    const int   *page_table; // [slots][max_pages]
    int          max_pages;
    const void  *kv_pages;       // this layer's region of the pool: f32 values, or f16 when kv_f16
    long long    page_elems;     // K/V values of one page in one layer: [K|V][kv head][token][d_head]
    int          n_pages;        // pages in the pool (bounds check)
    int          kv_f16;         // 1: the pool holds f16 values
    unsigned int *fault;         // device fault word
    int          layer, n_heads, n_kv, d_head, page_tokens;
    int          split_tokens;   // multiple of page_tokens
    int          n_splits;       // gridDim.x
    int          q_chunk;        // queries per shared-memory chunk of a prefill group (>= 1)
    int          grouped;        // 1: a session's consecutive columns share K / V loads
    int          q_block;        // queries per leader of a group (1..32)
    int          chunk_tokens;   // decode kernel: context tokens per CTA (set by attention_launch)
    // persistent tensor-core variant (f16 pools, steps of >= tc_min_cols columns);
    // the work plan is step metadata written by the host
    int          tc_min_cols;    // 0: never
    const int   *order;          // [B] live columns, longest context first
    const int   *chunk_pfx;      // [B+1] prefix sums of their chunk counts
    const int   *attn_n;         // [1] live columns
    const int   *attn_chunk;     // [1] context tokens per work item (multiple of 64)
    int         *work;           // [2 * layers] work-queue counters, zero between launches
    int          max_cols;       // capacity of order / chunk_pfx (the engine's max_batch)
    float        scale;          // 1/sqrt(d_head)
    float       *part;           // scratch [ncol][n_heads][n_splits][d_head + 2]
    int         *counters;       // scratch [ncol][n_kv], zero between launches
};

// Scratch floats / ints attention needs for ncol columns.
inline size_t attn_part_floats(int ncol, int n_heads, int n_splits, int d_head) {
    return (size_t)ncol * n_heads * n_splits * (d_head + 2);
}

// Dynamic shared memory one CTA needs (K and V tiles of kvb-byte values,
// queries, scores) with q_chunk queries per chunk.
size_t attention_smem_bytes(int d_head, int group, int split_tokens, int q_chunk, int kvb);
// Queries per chunk for engines whose steps carry prefill groups: about 6 KB
// of query and score tiles (decode-only engines use 1).
int attention_q_chunk(int d_head, int group, int split_tokens);
#define CMOLCU_ATTN_SMEM_MAX (200 * 1024)

cudaError_t attention_launch(const AttnArgs &a, int ncol, cudaStream_t st, bool pdl);
