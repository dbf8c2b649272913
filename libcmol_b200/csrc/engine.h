// engine.h — one GPU's decode engine (C++ interface, no CUDA types).
//
// Owns the uploaded model, the paged KV pool, per-slot sampler state and the
// activation buffers, and runs one decode step for a batch of columns: each
// column is one session contributing one token (its next prompt token, or
// the token it sampled last).  The step is captured once per batch-size
// bucket into a CUDA graph and replayed.  The host side that decides which
// sessions run (the batcher) lives in api.cpp.
#pragma once
#include <stdint.h>

#include <atomic>
#include <vector>

#include "host_model.h"

namespace cmolrt {

struct EngineOptions {
    int   max_batch = 4;       // columns per step
    int   max_slots = 4;       // sessions (slots) with page tables
    int   max_ctx = 2048;      // tokens per session
    int   page_tokens = 16;
    float kv_pool_frac = 0.85f;
    bool  use_graphs = true;
    int   split_tokens = 64;   // attention context split (tokens per work item)
    int   max_group = 1;       // most columns of one session in a step (prefill chunk)
    bool  kv_f16 = false;      // KV pool in f16 (values rounded to nearest on write) instead of f32
};

struct SamplerParams {
    float    temperature = 0.f, top_p = 1.f, repeat_penalty = 1.f;
    int      top_k = 0;
    int      eos = -1;
    uint64_t rng[4] = {0, 0, 0, 0};
    int      ring[128];
    int      ring_fill = 0, ring_head = 0;
};

struct StepColumn {
    int token;
    int pos;        // position the token is written at
    int slot;
    int sample;     // 1: run the sampler on this column's logits
};

struct PageUpdate {
    int slot, index, page;
};

struct EngineStats {
    long long steps = 0, tokens = 0, sampled = 0;
    double    step_ms_total = 0, step_ms_last = 0;
    long long decode_steps = 0;      // steps in which every column sampled
    double    decode_ms = 0;         // device time of those steps
    int       launches_per_step = 0;
    long long graph_steps = 0;
};

class Engine {
  public:
    // Returns nullptr and sets *err (cmol_err_t) on failure.
    static Engine *create(int device, const HostModel &m, const EngineOptions &o, int *err, char *msg, int msg_len);
    ~Engine();

    int  device() const { return device_; }
    int  n_pages() const { return n_pages_; }
    int  page_tokens() const { return opt_.page_tokens; }
    int  max_pages_per_slot() const { return max_pages_; }
    int  max_batch() const { return opt_.max_batch; }
    int  max_pages() const { return max_pages_; }
    const EngineOptions &options() const { return opt_; }
    int  vocab() const { return vocab_; }
    long long weight_bytes_per_step() const { return weight_bytes_; }
    long long kv_bytes_per_token() const { return kv_bytes_per_token_; }

    // Writes the sampler state of `slot` (async on the engine stream).
    int set_sampler(int slot, const SamplerParams &p);

    // Runs one step.  cols.size() <= max_batch.  Page updates are applied
    // before the step.  out_ids[i] receives the sampled token of column i
    // (undefined for columns with sample == 0).  When logits_out is not
    // NULL the logits of every column are copied there ([ncol][vocab]).
    // Returns 0, or -1 with a message in last_error().
    int step(const std::vector<StepColumn> &cols, const std::vector<PageUpdate> &upd,
             int32_t *out_ids, float *logits_out);

    // Device time of the GEMV launches of one decode step replayed alone
    // (graph, CUDA events); bytes = GGUF bytes of all matrices streamed.
    int gemv_sweep(int reps, double *ms_per_pass, long long *bytes_per_pass, int *launches_per_pass);

    // One kernel class of the widest step since the last reset_stats (the
    // latest of equal width), replayed alone `reps` times from a
    // CUDA graph (device time per pass by CUDA events on the engine stream):
    //   what 0: its weight products at its width (columns marked inactive,
    //           so no KV is written); bytes = GGUF bytes of every matrix,
    //           flops = 2 * weights * live columns;
    //   what 1: its attention launches over the same sessions, positions and
    //           pages (read-only on the KV cache); bytes = the K and V bytes
    //           those positions read, flops = 4 * heads * d_head * tokens.
    int kernel_sweep(int what, int reps, double *ms_per_pass, long long *bytes_per_pass, double *flops_per_pass,
                     int *launches_per_pass);

    const char *last_error() const { return err_; }
    // Fault-path test hook: the next step carries a planted error that the
    // device checks catch and skip (1: column 0's token id past the
    // vocabulary; 2: a page-table update naming a page outside the pool;
    // 3: the step-begin kernel's bounded wait runs out).
    void inject_fault(int kind) { inject_.store(kind); }
    // Session KV snapshots (multi-turn reuse).  kv_pages_copy moves pages
    // pages[0..n) of every layer to host memory laid out [layer][page][page
    // bytes] (to_host) or back into those pages; set_page_row writes engine
    // slot lslot's page-table entries [0, n).  Both synchronous, on no engine
    // stream: the caller keeps the session idle meanwhile.
    int kv_pages_copy(const int *pages, int n, void *host, bool to_host);
    int set_page_row(int lslot, const int *pages, int n);
    long long kv_page_bytes() const;   // one page of one layer
    int n_layers() const;
    int max_ctx() const { return opt_.max_ctx; }
    bool kv_f16() const { return opt_.kv_f16; }
    // Bytes one step copies host -> device (its metadata) and device -> host
    // (sampled ids and the fault word), logits excluded.
    long long h2d_bytes_per_step() const;
    long long d2h_bytes_per_step() const { return 4LL * (opt_.max_batch + 1); }
    // Device fault code of the last failed step (0 = none since load).
    unsigned int last_fault() const { return last_fault_; }
    EngineStats stats;
    void reset_stats() { stats = EngineStats(); last_n_ = 0; }
    unsigned int fault_code();   // device fault word (0 = none); clears it

    struct Impl;      // device state (engine.cu)

  private:
    Engine() = default;
    Impl *d = nullptr;
    int device_ = 0;
    EngineOptions opt_;
    int n_pages_ = 0, max_pages_ = 0, vocab_ = 0;
    long long weight_bytes_ = 0, kv_bytes_per_token_ = 0;
    std::atomic<int> inject_{0};
    std::vector<int> last_meta_;      // step metadata of the last step (host copy)
    int last_n_ = 0, last_bucket_ = 0;
    bool last_grouped_ = false;
    long long weight_values_ = 0;     // weights of every matrix one step streams
    unsigned int last_fault_ = 0;
    char err_[256] = {0};
    friend struct EngineBuilder;
};

}  // namespace cmolrt
