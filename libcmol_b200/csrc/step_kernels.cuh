// step_kernels.cuh — the small kernels of a decode step: step begin
// (page-table updates + embedding lookup) and the sampler.
#pragma once
#include "common.cuh"
#include "qweight.cuh"
#include "gemv.cuh"

#define CMOLCU_REPEAT_BUF 128     // src/sampler.h:49 of the reference
#define CMOLCU_TOPK_MAX   512     // src/sampler.c:150

// Per-session sampler state, resident in device memory (one per slot).
struct SlotSampler {
    unsigned long long rng[4];     // xoshiro256** state (src/sampler.c:37-84)
    int   ring[CMOLCU_REPEAT_BUF]; // repeat window ring buffer (src/api.c:465-507)
    int   ring_head, ring_fill;
    float temperature, top_p, repeat_penalty;
    int   top_k;
    int   eos;                     // < 0: none
    int   pad[3];
};

// Step metadata written host -> device once per step.  All arrays hold
// max_batch entries; `ncol` columns are live.
struct StepMetaPtrs {
    int *token;      // [B] input token of the column
    int *pos;        // [B] position (< 0 inactive)
    int *slot;       // [B] session slot
    int *sample;     // [B] 1: sample a token from this column's logits
    int *n_upd;      // [1] page-table updates this step
    int *upd;        // [3B] (slot, page index, page id) triples
    int *order;      // [B] live columns, longest context first (attention work order)
    int *chunk_pfx;  // [B+1] prefix sums of their attention chunk counts
    int *attn_n;     // [1] live columns
    int *attn_chunk; // [1] context tokens per attention work item
    int *stall;      // [1] 1: k_step_begin waits on a barrier nothing arrives on (fault-path test)
};

struct StepBeginArgs {
    StepMetaPtrs meta;
    int         *page_table;   // [slots][max_pages]
    int          max_pages;
    int          max_slots;
    int          n_pages;      // pages in the pool
    QWeight      embd;         // [vocab x d_model]
    float       *x;            // [B][d_model]
    int          d_model;
    unsigned int *fault;       // device fault word
};

struct SampleArgs {
    StepMetaPtrs meta;
    float       *logits;       // [B][vocab], modified in place
    int          vocab;
    SlotSampler *slots;
    int         *out_ids;      // [B]
    unsigned int *fault;       // device fault word
};

// Per-head RMSNorm of q and k (optional attn_q_norm / attn_k_norm, shared
// [d_head] weights, src/attn.c:62-80), then RoPE and the KV append, for
// models that carry QK-norm tensors.  One warp per head.
struct QkNormArgs {
    const float *qkv;  long long qkv_ld;   // raw projections [ncol][D + 2*KVD]
    float       *q_out; long long q_ld;
    const float *q_norm, *k_norm;          // NULL = no norm for that side
    float        eps;
    EpiQKV       e;
};

cudaError_t qknorm_launch(const QkNormArgs &a, int ncol, int n_heads, cudaStream_t st, bool pdl);

cudaError_t step_begin_launch(const StepBeginArgs &a, int ncol, cudaStream_t st, bool pdl);
cudaError_t sample_launch(const SampleArgs &a, int ncol, cudaStream_t st, bool pdl);
