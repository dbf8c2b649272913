// decode_step.cuh — the persistent decode-step kernel.
//
// One launch runs every layer of one decode step for up to NC columns
// (sessions): one CTA per SM, all resident at once (cooperative launch),
// walking a table of phases
//
//   per layer:  QKV   RMSNorm + q|k|v rows + RoPE + KV append     (GEMV)
//               ATTN  split-context GQA attention items             (attention_item.cuh)
//               WO    attention output . wo, += residual            (GEMV)
//               GU    RMSNorm + gate|up rows + SwiGLU               (GEMV)
//               DOWN  h . down, += residual                          (GEMV)
//   then        HEAD  RMSNorm + LM head                              (GEMV)
//
// with a grid barrier between consecutive phases (bounded spin on a global
// counter).  Weights do not depend on the activations, so the producer
// warp of each CTA walks the whole step's weight schedule — its rows of
// every GEMV phase, in phase order — and keeps a ring of shared-memory
// slots full with cp.async.bulk copies, running ahead across the barriers.
// The eight consumer warps stage each phase's activations after the
// barrier, consume the slots in the same order, and write the epilogue.
// The per-phase work of a small model is a few KB per SM, so the step is
// bounded by the barrier chain, not by bandwidth; the ring hides the HBM
// latency of the weights completely.
//
// The arithmetic is that of k_gemv (gemv.cuh) and k_attn (attention.cu):
// the same chunk_math, the same epilogues, the same attention item.
#pragma once
#include "attention.cuh"
#include "gemv.cuh"

enum : int { DS_GEMV = 0, DS_ATTN = 1 };

struct DsPhase {
    int      kind;          // DS_GEMV / DS_ATTN
    int      epi;           // EPI_* of a GEMV phase
    GemvArgs g;             // weight, x, norm, y, QKV epilogue, stage geometry (pc.po, pc.sb, pc.rows_per_cta)
    int      layer;         // attention layer
};

#define DS_MAX_SLOTS 12
#define DS_MAX_NC 4

struct DsArgs {
    const DsPhase *phases;
    int            n_phases;
    int            ncol;             // active columns this launch (<= NC)
    AttnArgs       attn;             // attention template (layer set per phase)
    unsigned int  *sync_count;       // grid barrier counter, zeroed before the launch
    unsigned int  *fault;
    int            nslot;            // ring slots
    int            slot_bytes;       // bytes per slot (multiple of 128)
    int            union_bytes;      // activation staging / attention region
    int            pages_bytes;      // page-table rows of the columns
    const float2  *rope_cs;          // [pos][d_head / 2] (cos, sin)
    unsigned long long *trace;       // optional: CTA 0 timestamps [2 * n_phases + 1] (ns, %globaltimer)
};

// Host side.
struct DsPlan {
    int    nc = 0;                   // template column count
    int    nslot = 0, slot_bytes = 0, union_bytes = 0, pages_bytes = 0;
    size_t smem = 0;
    int    grid = 0;
};

// Shared-memory plan for `phases` at nc columns; false if it cannot fit.
bool ds_plan(const DsPhase *phases_host, int n_phases, int nc, int d_head, int G, int split_tokens, int max_pages,
             DsPlan &plan);
// Rows of each GEMV phase per CTA for a grid of `grid` CTAs (fills pc.rows_per_cta, pc.po, pc.sb).
void ds_partition(DsPhase *phases_host, int n_phases, int grid);
cudaError_t ds_launch(const DsArgs &a, const DsPlan &plan, int d_head, cudaStream_t st, bool pdl);
