// engine.cu — one GPU's decode engine (see engine.h).
#include "engine.h"

#include <math.h>
#include <stdarg.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "attention.cuh"
#include "gemm_tc.cuh"
#include "gemv_launch.cuh"
#include "step_kernels.cuh"

namespace cmolrt {

namespace {

// A device weight plus the allocation backing it.
struct DevWeight {
    QWeight q = {};
    void   *base = nullptr;
};

struct Layer {
    DevWeight qkv;              // fused [D + 2*KVD] rows when q/k/v share a dtype
    DevWeight q, k, v;          // otherwise separate
    bool      fused_qkv = false;
    DevWeight wo, gu, down;     // gu: interleaved gate/up rows
    float    *attn_norm = nullptr, *ffn_norm = nullptr;
    float    *q_norm = nullptr, *k_norm = nullptr;
};

}  // namespace

struct Engine::Impl {
    HParams             hp;
    std::vector<Layer>  layers;
    DevWeight           embd, head;       // head.base == nullptr when tied
    float              *out_norm = nullptr;
    float2             *rope_cs = nullptr;
    void               *kv_pages = nullptr;   // f32 or f16 values (EngineOptions::kv_f16)
    long long           page_elems = 0;       // K/V values per page
    int                *page_table = nullptr;
    SlotSampler        *slots = nullptr;
    // step metadata: device block and pinned mirror (same layout)
    int                *meta_dev = nullptr, *meta_host = nullptr;
    size_t              meta_ints = 0;
    StepMetaPtrs        meta = {};
    int                *out_dev = nullptr, *out_host = nullptr;
    // activations
    float *x = nullptr, *qbuf = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr, *qkvbuf = nullptr;
    float *part = nullptr;
    int   *counters = nullptr;
    int   *work = nullptr;          // [2 * layers] attention work-queue counters
    unsigned int *fault = nullptr;
    int    n_splits = 1;
    int    attn_qc = 1;        // attention queries per chunk of a prefill group
    int    attn_grouped = 1;   // CMOLCU_ATTN_GROUP=0: every column loads its own K / V
    int    attn_qb = 8;        // queries per group leader (CMOLCU_ATTN_QB; 8 measured best)
    long long n_pages = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t  ev0 = nullptr, ev1 = nullptr;
    std::map<int, cudaGraphExec_t> graphs;
    std::vector<void *> allocs;
    int launches = 0;
    // tensor-core matmul for steps of >= tc_min_cols columns (gemm_tc.cuh)
    TcScratch     tc = {};
    bool          tc_ok = false;
    int           tc_min_cols = 16;
};

static void set_msg(char *dst, int n, const char *fmt, ...) {
    if (!dst || n <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(dst, (size_t)n, fmt, ap);
    va_end(ap);
}

struct EngineBuilder {
    Engine *e;
    Engine::Impl *d;
    char *msg;
    int msg_len;

    // All set-up traffic goes through the engine stream: the engine's kernels
    // run on a non-blocking stream, which does not order itself after work on
    // the legacy default stream.
    template <typename T>
    T *dalloc(size_t count, bool zero = true) {
        void *p = nullptr;
        if (cudaMalloc(&p, count * sizeof(T) + 16) != cudaSuccess) return nullptr;
        d->allocs.push_back(p);
        if (zero && (cudaMemsetAsync(p, 0, count * sizeof(T) + 16, d->stream) != cudaSuccess ||
                     cudaStreamSynchronize(d->stream) != cudaSuccess))
            return nullptr;
        return (T *)p;
    }

    // Upload `rows` GGUF rows of dtype dt, length k, into padded planes.
    bool upload(DevWeight &w, const uint8_t *rows_host, int dt, int rows, int k) {
        if (!qw_nplanes(dt) || k % dt_block_values(dt) || k % 16) {
            set_msg(msg, msg_len, "unsupported weight dtype %d / k %d", dt, k);
            return false;
        }
        QWeight q = {};
        const size_t tot = qw_layout(q, dt, rows, k, qw_default_kc(dt, k));
        uint8_t *base = dalloc<uint8_t>(tot);
        if (!base) { set_msg(msg, msg_len, "out of device memory (weights)"); return false; }
        for (int i = 0; i < q.nplanes; i++) q.p[i] = base + (uintptr_t)q.p[i];
        void *tmp = nullptr;
        cudaError_t err = cudaMalloc(&tmp, q.bytes);
        if (err == cudaSuccess) err = cudaMemcpyAsync(tmp, rows_host, q.bytes, cudaMemcpyHostToDevice, d->stream);
        if (err == cudaSuccess) err = repack_launch((const uint8_t *)tmp, q, d->stream);
        if (err == cudaSuccess) err = cudaStreamSynchronize(d->stream);
        if (tmp) cudaFree(tmp);
        if (err != cudaSuccess) { set_msg(msg, msg_len, "weight upload: %s", cudaGetErrorString(err)); return false; }
        w.q = q;
        w.base = base;
        return true;
    }

    float *upload_f32(const HTensor *t, int n) {
        if (!t || t->dtype != 0 || t->nbytes < (size_t)n * 4) return nullptr;
        float *p = dalloc<float>((size_t)n);
        if (!p) return nullptr;
        if (cudaMemcpyAsync(p, t->data, (size_t)n * 4, cudaMemcpyHostToDevice, d->stream) != cudaSuccess ||
            cudaStreamSynchronize(d->stream) != cudaSuccess)
            return nullptr;
        return p;
    }
};

// Scratch of the tensor-core matmul, sized for the largest weight at
// max_batch columns.  Steps of at least tc_min_cols columns use it for every
// weight in a format it handles (Q4_K, Q8_0, Q4_0, Q5_0); the rest, and
// smaller steps, use the exact f32 GEMV.  CMOLCU_TC_MIN_COLS overrides the
// threshold (1 forces the tensor cores for every step).
static void build_tensor_core_path(Engine *e, Engine::Impl *d, EngineBuilder &b) {
    const EngineOptions &o = e->options();
    const char *env = getenv("CMOLCU_TC_MIN_COLS");
    if (env && atoi(env) > 0) d->tc_min_cols = atoi(env);
    if (o.max_batch < d->tc_min_cols) return;
    size_t xs = 0, part = 0;
    int rbs = 0;
    auto need = [&](const DevWeight &w) {
        if (!w.base || !tc_supported(w.q.dtype)) return;
        size_t a = 0, p = 0;
        int r = 0;
        tc_scratch_need(w.q.rows, w.q.k, std::min(o.max_batch, TC_MAX_N), &a, &p, &r);
        xs = std::max(xs, a);
        part = std::max(part, p);
        rbs = std::max(rbs, r);
    };
    for (const Layer &ly : d->layers) {
        need(ly.qkv); need(ly.q); need(ly.k); need(ly.v);
        need(ly.wo); need(ly.gu); need(ly.down);
    }
    need(d->head.base ? d->head : d->embd);
    if (!xs) return;
    d->tc.xs = b.dalloc<uint16_t>(xs);
    d->tc.part = b.dalloc<float>(std::max<size_t>(part, 1));
    d->tc.part_floats = part;
    d->tc.counters = b.dalloc<int>((size_t)rbs);
    d->tc.max_row_blocks = rbs;
    d->tc_ok = d->tc.xs && d->tc.part && d->tc.counters;
    if (!d->tc_ok) cudaGetLastError();
}

Engine *Engine::create(int device, const HostModel &m, const EngineOptions &o, int *err, char *msg, int msg_len) {
    const HParams &hp = m.hp;
    *err = -4;  // CMOL_ERR_UNSUPPORTED
    if (cudaSetDevice(device) != cudaSuccess) { set_msg(msg, msg_len, "cannot use CUDA device %d", device); return nullptr; }
    if (hp.n_layers <= 0 || hp.d_model <= 0 || hp.n_heads <= 0 || hp.d_ffn <= 0 || hp.vocab_size <= 0 ||
        hp.n_kv_heads <= 0 || hp.d_model % hp.n_heads || hp.n_heads % hp.n_kv_heads) {
        *err = -3;
        set_msg(msg, msg_len, "bad hyperparameters");
        return nullptr;
    }
    const int D = hp.d_model, F = hp.d_ffn, V = hp.vocab_size, L = hp.n_layers;
    const int hd = hp.d_head, nkv = hp.n_kv_heads, KVD = nkv * hd;
    if (hd % 32 || hd > 256 || D > CMOLCU_GEMV_MAX_K || F > CMOLCU_GEMV_MAX_K) {
        set_msg(msg, msg_len, "unsupported shape (d_head %d, d_model %d, d_ffn %d)", hd, D, F);
        return nullptr;
    }
    Engine *e = new Engine();
    e->device_ = device;
    e->opt_ = o;
    // attention keeps a whole split of K and V in shared memory: shrink the
    // split (in whole pages) until it fits
    auto q_chunk = [&](int split) { return o.max_group > 1 ? attention_q_chunk(hd, hp.n_heads / nkv, split) : 1; };
    while (e->opt_.split_tokens > o.page_tokens &&
           attention_smem_bytes(hd, hp.n_heads / nkv, e->opt_.split_tokens, q_chunk(e->opt_.split_tokens),
                                o.kv_f16 ? 2 : 4) >
               CMOLCU_ATTN_SMEM_MAX)
        e->opt_.split_tokens -= o.page_tokens;
    e->vocab_ = V;
    Impl *d = new Impl();
    e->d = d;
    d->hp = hp;
    d->attn_qc = q_chunk(e->opt_.split_tokens);
    if (const char *v = getenv("CMOLCU_ATTN_GROUP")) d->attn_grouped = v[0] != '0';
    if (const char *v = getenv("CMOLCU_ATTN_QB")) d->attn_qb = std::max(1, std::min(32, atoi(v)));
    EngineBuilder b{e, d, msg, msg_len};
    auto fail = [&](int code) -> Engine * { *err = code; delete e; return nullptr; };

    if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(-1);
    cudaEventCreate(&d->ev0);
    cudaEventCreate(&d->ev1);

    // ---- weights ----------------------------------------------------------
    const HTensor *te = m.find("token_embd.weight");
    if (!te || te->dims[0] != D || te->dims[1] < V) { set_msg(msg, msg_len, "token_embd.weight missing or misshaped"); return fail(-3); }
    if (!b.upload(d->embd, te->data, te->dtype, V, D)) return fail(-4);
    long long wbytes = 0;
    const HTensor *th = m.find("output.weight");
    if (th) {
        if (th->dims[0] != D) { set_msg(msg, msg_len, "output.weight misshaped"); return fail(-3); }
        if (!b.upload(d->head, th->data, th->dtype, V, D)) return fail(-4);
        wbytes += (long long)d->head.q.bytes;
    } else {
        wbytes += (long long)d->embd.q.bytes;
    }
    d->out_norm = b.upload_f32(m.find("output_norm.weight"), D);
    if (!d->out_norm) { set_msg(msg, msg_len, "output_norm.weight missing"); return fail(-3); }

    d->layers.resize((size_t)L);
    std::vector<uint8_t> buf;
    for (int l = 0; l < L; l++) {
        Layer &ly = d->layers[(size_t)l];
        const HTensor *wq = m.blk(l, "attn_q.weight"), *wk = m.blk(l, "attn_k.weight"),
                      *wv = m.blk(l, "attn_v.weight"), *wo = m.blk(l, "attn_output.weight"),
                      *wg = m.blk(l, "ffn_gate.weight"), *wu = m.blk(l, "ffn_up.weight"),
                      *wd = m.blk(l, "ffn_down.weight");
        if (!wq || !wk || !wv || !wo || !wg || !wu || !wd) {
            set_msg(msg, msg_len, "layer %d: missing tensor", l);
            return fail(-3);
        }
        ly.attn_norm = b.upload_f32(m.blk(l, "attn_norm.weight"), D);
        ly.ffn_norm = b.upload_f32(m.blk(l, "ffn_norm.weight"), D);
        if (!ly.attn_norm || !ly.ffn_norm) { set_msg(msg, msg_len, "layer %d: missing norm", l); return fail(-3); }
        ly.q_norm = b.upload_f32(m.blk(l, "attn_q_norm.weight"), hd);
        ly.k_norm = b.upload_f32(m.blk(l, "attn_k_norm.weight"), hd);
        if (wq->dtype == wk->dtype && wk->dtype == wv->dtype) {
            size_t rq = dtype_row_bytes(wq->dtype, D);
            buf.resize(rq * (size_t)(D + 2 * KVD));
            memcpy(buf.data(), wq->data, rq * D);
            memcpy(buf.data() + rq * D, wk->data, rq * KVD);
            memcpy(buf.data() + rq * (D + KVD), wv->data, rq * KVD);
            if (!b.upload(ly.qkv, buf.data(), wq->dtype, D + 2 * KVD, D)) return fail(-4);
            ly.fused_qkv = true;
            wbytes += (long long)ly.qkv.q.bytes;
        } else {
            if (!b.upload(ly.q, wq->data, wq->dtype, D, D) || !b.upload(ly.k, wk->data, wk->dtype, KVD, D) ||
                !b.upload(ly.v, wv->data, wv->dtype, KVD, D))
                return fail(-4);
            wbytes += (long long)(ly.q.q.bytes + ly.k.q.bytes + ly.v.q.bytes);
        }
        if (!b.upload(ly.wo, wo->data, wo->dtype, D, D)) return fail(-4);
        if (wg->dtype != wu->dtype) { set_msg(msg, msg_len, "layer %d: gate/up dtypes differ", l); return fail(-4); }
        {
            size_t rg = dtype_row_bytes(wg->dtype, D);
            buf.resize(rg * (size_t)(2 * F));
            for (int i = 0; i < F; i++) {   // rows 2i = gate_i, 2i+1 = up_i
                memcpy(buf.data() + rg * (2 * (size_t)i), wg->data + rg * i, rg);
                memcpy(buf.data() + rg * (2 * (size_t)i + 1), wu->data + rg * i, rg);
            }
            if (!b.upload(ly.gu, buf.data(), wg->dtype, 2 * F, D)) return fail(-4);
        }
        if (!b.upload(ly.down, wd->data, wd->dtype, D, F)) return fail(-4);
        wbytes += (long long)(ly.wo.q.bytes + ly.gu.q.bytes + ly.down.q.bytes);
    }
    e->weight_bytes_ = wbytes;
    {
        long long wv = (long long)V * D;   // the LM head (the embedding when tied)
        for (const Layer &ly : d->layers) {
            const DevWeight *ws[] = {&ly.qkv, &ly.q, &ly.k, &ly.v, &ly.wo, &ly.gu, &ly.down};
            for (const DevWeight *w : ws)
                if (w->base) wv += (long long)w->q.rows * w->q.k;
        }
        e->weight_values_ = wv;
    }
    std::vector<uint8_t>().swap(buf);

    // ---- RoPE table: theta = pos / base^(2i/d_head), src/model.c:146-148 ----
    {
        const int ctx = o.max_ctx;
        std::vector<float2> cs((size_t)ctx * (hd / 2));
        for (int p = 0; p < ctx; p++)
            for (int i = 0; i < hd / 2; i++) {
                float theta = (float)p / powf(hp.rope_freq_base, (float)(2 * i) / (float)hd);
                cs[(size_t)p * (hd / 2) + i] = make_float2(cosf(theta), sinf(theta));
            }
        d->rope_cs = b.dalloc<float2>(cs.size());
        if (!d->rope_cs ||
            cudaMemcpyAsync(d->rope_cs, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice, d->stream) != cudaSuccess ||
            cudaStreamSynchronize(d->stream) != cudaSuccess)
            return fail(-1);
    }

    // ---- activations, metadata, sampler state ------------------------------
    const int B = o.max_batch;
    d->x = b.dalloc<float>((size_t)B * D);
    d->qbuf = b.dalloc<float>((size_t)B * D);
    d->attn = b.dalloc<float>((size_t)B * D);
    d->h = b.dalloc<float>((size_t)B * F);
    d->logits = b.dalloc<float>((size_t)B * V);
    d->qkvbuf = b.dalloc<float>((size_t)B * (D + 2 * KVD));
    d->n_splits = (o.max_ctx + e->opt_.split_tokens - 1) / e->opt_.split_tokens;
    d->part = b.dalloc<float>(attn_part_floats(B, hp.n_heads, d->n_splits, hd));
    d->counters = b.dalloc<int>((size_t)B * nkv);

    d->slots = b.dalloc<SlotSampler>((size_t)o.max_slots);
    d->meta_ints = (size_t)4 * B + 1 + 3 * (size_t)B + B + (B + 1) + 3;
    d->meta_dev = b.dalloc<int>(d->meta_ints);
    d->out_dev = b.dalloc<int>((size_t)B + 1);   // + the fault word, read back with the ids
    d->fault = reinterpret_cast<unsigned int *>(d->out_dev + B);
    if (!d->x || !d->qbuf || !d->attn || !d->h || !d->logits || !d->qkvbuf || !d->part || !d->counters ||
        !d->fault || !d->slots || !d->meta_dev || !d->out_dev) {
        set_msg(msg, msg_len, "out of device memory (activations)");
        return fail(-1);
    }
    if (cudaMallocHost(&d->meta_host, d->meta_ints * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&d->out_host, ((size_t)B + 1) * sizeof(int)) != cudaSuccess)
        return fail(-1);
    d->meta.token = d->meta_dev;
    d->meta.pos = d->meta_dev + B;
    d->meta.slot = d->meta_dev + 2 * B;
    d->meta.sample = d->meta_dev + 3 * B;
    d->meta.n_upd = d->meta_dev + 4 * B;
    d->meta.upd = d->meta_dev + 4 * B + 1;
    d->meta.order = d->meta_dev + 7 * B + 1;
    d->meta.chunk_pfx = d->meta_dev + 8 * B + 1;
    d->meta.attn_n = d->meta_dev + 9 * B + 2;
    d->meta.attn_chunk = d->meta_dev + 9 * B + 3;
    d->meta.stall = d->meta_dev + 9 * B + 4;
    d->work = b.dalloc<int>((size_t)2 * L);
    if (!d->work) return fail(-1);

    // ---- KV page pool ------------------------------------------------------
    const int P = o.page_tokens;
    e->max_pages_ = (o.max_ctx + P - 1) / P;
    const int kvb = o.kv_f16 ? 2 : 4;
    // The pool is one region per layer: layer l's K and V of page pg start at
    // kv_pages + (l * n_pages + pg) * page_elems values, as [kv head][K|V]
    // [token][d_head], so one kv head's K and V of a page are one contiguous
    // block (32 KB for 64-token f16 pages of d_head 128): attention reads the
    // pool in blocks that size, since scattered reads of small blocks stream
    // far below the HBM rate (4 KB blocks measured at about a quarter of it).
    d->page_elems = (long long)2 * nkv * P * hd;
    e->kv_bytes_per_token_ = (long long)L * 2 * KVD * kvb;
    d->page_table = b.dalloc<int>((size_t)o.max_slots * e->max_pages_);
    if (!d->page_table) return fail(-1);
    {
        size_t fr = 0, tot = 0;
        cudaMemGetInfo(&fr, &tot);
        const size_t page_bytes = (size_t)L * d->page_elems * kvb;     // a page of every layer
        long long want = (long long)o.max_slots * e->max_pages_;
        long long fit = (long long)((double)fr * o.kv_pool_frac / (double)page_bytes);
        long long n = want < fit ? want : fit;
        if (n < e->max_pages_) { set_msg(msg, msg_len, "KV pool: not enough device memory"); return fail(-1); }
        d->kv_pages = b.dalloc<uint8_t>((size_t)n * page_bytes, false);
        if (!d->kv_pages) { set_msg(msg, msg_len, "KV pool allocation failed"); return fail(-1); }
        e->n_pages_ = (int)n;
        d->n_pages = n;
    }
    build_tensor_core_path(e, d, b);
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(-1);
    *err = 0;
    return e;
}

Engine::~Engine() {
    if (!d) return;
    cudaSetDevice(device_);
    if (d->stream) cudaStreamSynchronize(d->stream);
    for (auto &kv : d->graphs) cudaGraphExecDestroy(kv.second);
    for (void *p : d->allocs) cudaFree(p);
    if (d->meta_host) cudaFreeHost(d->meta_host);
    if (d->out_host) cudaFreeHost(d->out_host);
    if (d->ev0) cudaEventDestroy(d->ev0);
    if (d->ev1) cudaEventDestroy(d->ev1);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
}

unsigned int Engine::fault_code() {
    unsigned int v = 0;
    cudaSetDevice(device_);
    cudaMemcpyAsync(&v, d->fault, sizeof v, cudaMemcpyDeviceToHost, d->stream);
    if (cudaStreamSynchronize(d->stream) == cudaSuccess && v) {
        cudaMemsetAsync(d->fault, 0, sizeof v, d->stream);
        cudaStreamSynchronize(d->stream);
    }
    return v;
}


int Engine::set_sampler(int slot, const SamplerParams &p) {
    if (slot < 0 || slot >= opt_.max_slots) return -1;
    SlotSampler s = {};
    for (int i = 0; i < 4; i++) s.rng[i] = p.rng[i];
    for (int i = 0; i < CMOLCU_REPEAT_BUF; i++) s.ring[i] = p.ring[i];
    s.ring_head = p.ring_head;
    s.ring_fill = p.ring_fill;
    s.temperature = p.temperature;
    s.top_p = p.top_p;
    s.repeat_penalty = p.repeat_penalty;
    s.top_k = p.top_k;
    s.eos = p.eos;
    cudaSetDevice(device_);
    // synchronous: the caller's stack copy must stay valid until the copy is done
    if (cudaMemcpyAsync(d->slots + slot, &s, sizeof s, cudaMemcpyHostToDevice, d->stream) != cudaSuccess ||
        cudaStreamSynchronize(d->stream) != cudaSuccess) {
        snprintf(err_, sizeof err_, "set_sampler: copy failed");
        return -1;
    }
    return 0;
}

// One weight product of a step: the tensor cores when the step is wide
// enough and the format has a tensor-core path, else the f32 GEMV.
static cudaError_t step_matmul(Engine::Impl *d, const GemvArgs &a, int ncol, int epi, cudaStream_t st, bool pdl,
                               int &launches) {
    if (d->tc_ok && ncol >= d->tc_min_cols && tc_supported(a.w.dtype) && a.w.k % TC_KB == 0 && a.w.kc % TC_KB == 0) {
        // blocks of at most TC_MAX_N columns (one tensor-memory accumulator each)
        for (int c0 = 0; c0 < ncol; c0 += TC_MAX_N) {
            GemvArgs b = a;
            const int n = std::min(TC_MAX_N, ncol - c0);
            b.x = a.x + (long long)c0 * a.x_ld;
            b.y = a.y + (long long)c0 * a.y_ld;
            if (epi == EPI_QKV) {
                b.qkv.pos = a.qkv.pos + c0;
                if (a.qkv.slot) b.qkv.slot = a.qkv.slot + c0;
                else b.qkv.page_table = a.qkv.page_table + (long long)c0 * a.qkv.max_pages;
            }
            launches += 2;
            cudaError_t e = tc_matmul(b, n, epi, d->tc, st, pdl);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    launches += (ncol + 1) / 2;
    return gemv_launch_cols(a, ncol, epi, st, pdl);
}

// Layer l's region of the KV pool.
static void *kv_layer(const Engine::Impl *d, int l, const EngineOptions &o) {
    return static_cast<unsigned char *>(d->kv_pages) + (size_t)l * d->n_pages * d->page_elems * (o.kv_f16 ? 2 : 4);
}

long long Engine::kv_page_bytes() const { return d ? d->page_elems * (opt_.kv_f16 ? 2 : 4) : 0; }
int Engine::n_layers() const { return d ? d->hp.n_layers : 0; }

int Engine::kv_pages_copy(const int *pages, int n, void *host, bool to_host) {
    if (!d || n < 0 || (n > 0 && (!pages || !host))) return -1;
    cudaSetDevice(device_);
    const size_t pb = (size_t)kv_page_bytes();
    unsigned char *h = static_cast<unsigned char *>(host);
    for (int i = 0; i < n; i++)
        if (pages[i] < 0 || pages[i] >= n_pages_) {
            snprintf(err_, sizeof err_, "kv copy: page %d outside the pool", pages[i]);
            return -1;
        }
    for (int l = 0; l < d->hp.n_layers; l++) {
        unsigned char *base = static_cast<unsigned char *>(kv_layer(d, l, opt_));
        for (int i = 0; i < n; i++) {
            unsigned char *dv = base + (size_t)pages[i] * pb;
            unsigned char *hv = h + ((size_t)l * n + i) * pb;
            const cudaError_t e = to_host ? cudaMemcpy(hv, dv, pb, cudaMemcpyDeviceToHost)
                                          : cudaMemcpy(dv, hv, pb, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                snprintf(err_, sizeof err_, "kv copy: %s", cudaGetErrorString(e));
                return -1;
            }
        }
    }
    return 0;
}

int Engine::set_page_row(int lslot, const int *pages, int n) {
    if (!d || lslot < 0 || lslot >= opt_.max_slots || n < 0 || n > max_pages_ || (n > 0 && !pages)) return -1;
    if (n == 0) return 0;
    cudaSetDevice(device_);
    const cudaError_t e =
        cudaMemcpy(d->page_table + (size_t)lslot * max_pages_, pages, (size_t)n * sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        snprintf(err_, sizeof err_, "page table: %s", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// What record_step records: the whole step, only its weight products, or
// only its attention launches (the last two for the kernel sweeps).
enum { REC_FULL = 0, REC_MATMUL = 1, REC_ATTN = 2 };

// Records the kernels of one step for `ncol` columns on the engine stream.
static cudaError_t record_step(Engine::Impl *d, const EngineOptions &o, int ncol, int max_pages, int &launches,
                               int only = REC_FULL, bool grouped = false) {
    const bool gemv_only = only == REC_MATMUL;
    const bool mm = only != REC_ATTN;
    const HParams &hp = d->hp;
    const int D = hp.d_model, F = hp.d_ffn, V = hp.vocab_size;
    const int hd = hp.d_head, nkv = hp.n_kv_heads, KVD = nkv * hd;
    const cudaStream_t st = d->stream;
    const bool pdl = true;
    cudaError_t e;
    launches = 0;

    StepBeginArgs sb = {};
    sb.meta = d->meta;
    sb.page_table = d->page_table;
    sb.max_pages = max_pages;
    sb.max_slots = o.max_slots;
    sb.n_pages = (int)d->n_pages;
    sb.embd = d->embd.q;
    sb.x = d->x;
    sb.d_model = D;
    sb.fault = d->fault;
    if (only == REC_FULL) {
        if ((e = step_begin_launch(sb, ncol, st, false)) != cudaSuccess) return e;
        launches++;
    }

    GemvArgs g = {};
    g.x_inc = 1;
    g.y_inc = 1;
    g.eps = hp.rms_norm_eps;
    g.fault = d->fault;
    for (int l = 0; l < hp.n_layers; l++) {
        const Layer &ly = d->layers[(size_t)l];
        const bool nope = hp.no_rope_layer_interval > 0 && (l + 1) % hp.no_rope_layer_interval == 0;
        const bool qkn = ly.q_norm || ly.k_norm;
        // --- Q/K/V projection (+ RoPE + KV append) --------------------------
        EpiQKV q = {};
        q.d_model = D; q.kv_dim = KVD; q.d_head = hd; q.n_kv = nkv; q.page_tokens = o.page_tokens;
        q.layer = l; q.rope = nope ? 0 : 1; q.rope_cs = d->rope_cs;
        q.pos = d->meta.pos; q.slot = d->meta.slot; q.page_table = d->page_table; q.max_pages = max_pages;
        q.kv_pages = kv_layer(d, l, o); q.page_elems = d->page_elems; q.n_pages = (int)d->n_pages;
        q.kv_f16 = o.kv_f16 ? 1 : 0;
        auto qkv_part = [&](const DevWeight &w, int row_base) -> cudaError_t {
            GemvArgs a = g;
            a.w = w.q;
            a.x = d->x; a.x_ld = D;
            a.norm_w = ly.attn_norm;
            if (qkn) {   // raw projections; norm + RoPE + KV append in the next kernel
                a.y = d->qkvbuf + row_base; a.y_ld = D + 2 * KVD;
                return step_matmul(d, a, ncol, EPI_STORE, st, pdl, launches);
            }
            a.y = d->qbuf; a.y_ld = D;
            a.qkv = q;
            a.qkv.row_base = row_base;
            return step_matmul(d, a, ncol, EPI_QKV, st, pdl, launches);
        };
        if (!mm) {
        } else if (ly.fused_qkv) {
            if ((e = qkv_part(ly.qkv, 0)) != cudaSuccess) return e;
        } else {
            if ((e = qkv_part(ly.q, 0)) != cudaSuccess) return e;
            if ((e = qkv_part(ly.k, D)) != cudaSuccess) return e;
            if ((e = qkv_part(ly.v, D + KVD)) != cudaSuccess) return e;
        }
        if (qkn && only == REC_FULL) {
            QkNormArgs qa = {};
            qa.qkv = d->qkvbuf; qa.qkv_ld = D + 2 * KVD;
            qa.q_out = d->qbuf; qa.q_ld = D;
            qa.q_norm = ly.q_norm; qa.k_norm = ly.k_norm; qa.eps = hp.rms_norm_eps;
            qa.e = q;
            if ((e = qknorm_launch(qa, ncol, hp.n_heads, st, pdl)) != cudaSuccess) return e;
            launches++;
        }
        // --- attention -------------------------------------------------------
        AttnArgs at = {};
        at.q = d->qbuf; at.q_ld = D;
        at.out = d->attn; at.out_ld = D;
        at.pos = d->meta.pos; at.slot = d->meta.slot;
        at.page_table = d->page_table; at.max_pages = max_pages;
        at.kv_pages = kv_layer(d, l, o); at.page_elems = d->page_elems; at.n_pages = (int)d->n_pages;
        at.kv_f16 = o.kv_f16 ? 1 : 0;
        at.fault = d->fault;
        at.layer = l; at.n_heads = hp.n_heads; at.n_kv = nkv; at.d_head = hd; at.page_tokens = o.page_tokens;
        at.split_tokens = o.split_tokens; at.n_splits = d->n_splits; at.q_chunk = d->attn_qc; at.grouped = grouped;
        at.q_block = d->attn_qb;
        at.scale = 1.0f / sqrtf((float)hd);
        at.part = d->part; at.counters = d->counters;
        at.tc_min_cols = d->tc_min_cols;
        at.order = d->meta.order; at.chunk_pfx = d->meta.chunk_pfx;
        at.attn_n = d->meta.attn_n; at.attn_chunk = d->meta.attn_chunk;
        at.work = d->work; at.max_cols = o.max_batch;
        if (!gemv_only) {
            if ((e = attention_launch(at, ncol, st, pdl)) != cudaSuccess) return e;
            launches++;
        }
        if (!mm) continue;
        // --- output projection + residual -----------------------------------
        {
            GemvArgs a = g;
            a.w = ly.wo.q;
            a.x = d->attn; a.x_ld = D;
            a.y = d->x; a.y_ld = D;
            if ((e = step_matmul(d, a, ncol, EPI_RESID, st, pdl, launches)) != cudaSuccess) return e;
        }
        // --- FFN: norm + gate/up + SwiGLU, then down + residual --------------
        {
            GemvArgs a = g;
            a.w = ly.gu.q;
            a.x = d->x; a.x_ld = D;
            a.norm_w = ly.ffn_norm;
            a.y = d->h; a.y_ld = F;
            if ((e = step_matmul(d, a, ncol, EPI_SWIGLU, st, pdl, launches)) != cudaSuccess) return e;
        }
        {
            GemvArgs a = g;
            a.w = ly.down.q;
            a.x = d->h; a.x_ld = F;
            a.y = d->x; a.y_ld = D;
            if ((e = step_matmul(d, a, ncol, EPI_RESID, st, pdl, launches)) != cudaSuccess) return e;
        }
    }
    if (!mm) return cudaSuccess;
    // --- final norm + LM head, sampler ----------------------------------------
    {
        GemvArgs a = g;
        a.w = d->head.base ? d->head.q : d->embd.q;
        a.x = d->x; a.x_ld = D;
        a.norm_w = d->out_norm;
        a.y = d->logits; a.y_ld = V;
        if ((e = step_matmul(d, a, ncol, EPI_STORE, st, pdl, launches)) != cudaSuccess) return e;
    }
    if (gemv_only) return cudaSuccess;
    SampleArgs sa = {};
    sa.meta = d->meta;
    sa.logits = d->logits;
    sa.vocab = V;
    sa.slots = d->slots;
    sa.out_ids = d->out_dev;
    sa.fault = d->fault;
    if ((e = sample_launch(sa, ncol, st, pdl)) != cudaSuccess) return e;
    launches++;
    return cudaSuccess;
}

// Work plan of the persistent decode attention (attention_decode.cuh) in the
// step metadata: the live columns by context length, longest first; the
// chunk size, the largest power-of-two multiple of 64 tokens (up to 4096)
// that still gives about six (chunk, kv head) items per SM; and the prefix
// sums of the columns' chunk counts.
long long Engine::h2d_bytes_per_step() const { return d ? (long long)d->meta_ints * 4 : 0; }

static void attention_plan(int *m, const std::vector<StepColumn> &cols, int B, int n_kv, int page_tokens) {
    int *order = m + 7 * B + 1, *pfx = m + 8 * B + 1;
    int nl = 0;
    for (int i = 0; i < (int)cols.size(); i++)
        if (cols[i].pos >= 0) order[nl++] = i;
    std::stable_sort(order, order + nl, [&](int x, int y) { return cols[x].pos > cols[y].pos; });
    // CMOLCU_ATTN_ITEMS_PER_SM / CMOLCU_ATTN_CHUNK_MAX: measurement switches
    static const int per_sm = [] {
        const char *v = getenv("CMOLCU_ATTN_ITEMS_PER_SM");
        return v && atoi(v) > 0 ? atoi(v) : 6;
    }();
    static const int ch_max = [] {
        const char *v = getenv("CMOLCU_ATTN_CHUNK_MAX");
        const int c = v ? atoi(v) : 0;
        return c >= 64 && c <= 4096 && (c & (c - 1)) == 0 ? c : 4096;
    }();
    const long long target = (long long)per_sm * device_sm_count();
    auto items = [&](int c) {
        long long t = 0;
        for (int r = 0; r < nl; r++) t += cols[order[r]].pos / c + 1;
        return t * n_kv;
    };
    int ch = ch_max;                              // at most 256 pages an item (its page list in shared memory)
    while (ch > 256 * page_tokens) ch >>= 1;
    while (ch > 64 && items(ch) < target) ch >>= 1;
    pfx[0] = 0;
    for (int r = 0; r < nl; r++) pfx[r + 1] = pfx[r] + cols[order[r]].pos / ch + 1;
    m[9 * B + 2] = nl;
    m[9 * B + 3] = ch;
}

int Engine::step(const std::vector<StepColumn> &cols, const std::vector<PageUpdate> &upd, int32_t *out_ids,
                 float *logits_out) {
    const int n = (int)cols.size();
    const int B = opt_.max_batch;
    if (n <= 0 || n > B || (int)upd.size() > B) {
        snprintf(err_, sizeof err_, "step: bad batch (%d columns, %d page updates)", n, (int)upd.size());
        return -1;
    }
    cudaSetDevice(device_);
    // Steps of all engines on one device run one at a time: the persistent
    // step kernel's CTAs wait on one another, so two of its grids must never
    // share the device's SMs.
    static std::mutex dev_mu[64];
    std::unique_lock<std::mutex> dev_lock(dev_mu[device_ & 63]);
    int bucket = 1;
    while (bucket < n) bucket <<= 1;
    if (bucket > B) bucket = B;
    // a prefill group (consecutive positions of one session) selects the
    // step variant whose attention shares K / V loads within the group
    bool grouped = false;
    for (int i = 1; i < n && d->attn_grouped && !grouped; i++)
        grouped = cols[i].slot == cols[i - 1].slot && cols[i].pos == cols[i - 1].pos + 1 && cols[i - 1].pos >= 0;
    const int gkey = bucket * 2 + (grouped ? 1 : 0);
    int *m = d->meta_host;
    for (int i = 0; i < B; i++) {
        bool live = i < n;
        m[i] = live ? cols[i].token : 0;
        m[B + i] = live ? cols[i].pos : -1;
        m[2 * B + i] = live ? cols[i].slot : 0;
        m[3 * B + i] = live ? cols[i].sample : 0;
    }
    m[4 * B] = (int)upd.size();
    for (size_t u = 0; u < upd.size(); u++) {
        m[4 * B + 1 + 3 * u] = upd[u].slot;
        m[4 * B + 2 + 3 * u] = upd[u].index;
        m[4 * B + 3 + 3 * u] = upd[u].page;
    }
    // planted errors of the fault-path tests: kinds 1 and 2 are caught by the
    // bounds checks of k_step_begin, which record the code and skip the
    // access; kind 3 makes k_step_begin's bounded wait run out (code 7)
    attention_plan(m, cols, B, d->hp.n_kv_heads, opt_.page_tokens);
    const int inject = inject_.exchange(0);
    m[9 * B + 4] = inject == 3 ? 1 : 0;
    if (inject == 1) {
        m[0] = vocab_ + 3;
    } else if (inject == 2 && (int)upd.size() < B) {
        const int u = (int)upd.size();
        m[4 * B] = u + 1;
        m[4 * B + 1 + 3 * u] = cols[0].slot;
        m[4 * B + 2 + 3 * u] = 0;
        m[4 * B + 3 + 3 * u] = n_pages_ + 5;
    }
    if (n >= last_n_) {   // the kernel sweeps replay the widest step since the last stats reset
        last_meta_.assign(m, m + d->meta_ints);
        last_n_ = n;
        last_bucket_ = bucket;
        last_grouped_ = grouped;
    }
    cudaError_t e = cudaMemcpyAsync(d->meta_dev, d->meta_host, d->meta_ints * sizeof(int), cudaMemcpyHostToDevice,
                                    d->stream);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev0, d->stream);
    int launches = 0;
    if (e == cudaSuccess) {
        auto it = d->graphs.find(gkey);
        if (!opt_.use_graphs || it == d->graphs.end()) {
            // eager launches: always the first step of a bucket (sets kernel
            // attributes outside any capture), every step without graphs
            e = record_step(d, opt_, bucket, max_pages_, launches, REC_FULL, grouped);
            d->launches = launches;
            if (e == cudaSuccess && opt_.use_graphs) {
                // capture this bucket for the next steps (capture does not run)
                cudaGraph_t g = nullptr;
                cudaGraphExec_t ge = nullptr;
                int l2 = 0;
                e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal);
                if (e == cudaSuccess) {
                    cudaError_t re = record_step(d, opt_, bucket, max_pages_, l2, REC_FULL, grouped);
                    e = cudaStreamEndCapture(d->stream, &g);
                    if (re != cudaSuccess) e = re;
                }
                if (e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
                if (g) cudaGraphDestroy(g);
                if (e == cudaSuccess) d->graphs[gkey] = ge;
            }
        } else {
            e = cudaGraphLaunch(it->second, d->stream);
            if (e == cudaSuccess) stats.graph_steps++;
        }
    }
    if (e == cudaSuccess) e = cudaEventRecord(d->ev1, d->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d->out_host, d->out_dev, ((size_t)B + 1) * sizeof(int), cudaMemcpyDeviceToHost, d->stream);
    if (e == cudaSuccess && logits_out)
        e = cudaMemcpyAsync(logits_out, d->logits, (size_t)n * vocab_ * sizeof(float), cudaMemcpyDeviceToHost, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) {
        snprintf(err_, sizeof err_, "step: %s", cudaGetErrorString(e));
        return -1;
    }
    const unsigned int fault = (unsigned int)d->out_host[B];
    if (fault) {
        last_fault_ = fault;
        cudaMemsetAsync(d->fault, 0, sizeof(unsigned int), d->stream);
        // an abandoned step can leave attention split counters behind
        cudaMemsetAsync(d->counters, 0, (size_t)B * d->hp.n_kv_heads * sizeof(int), d->stream);
        cudaMemsetAsync(d->work, 0, (size_t)2 * d->hp.n_layers * sizeof(int), d->stream);
        cudaStreamSynchronize(d->stream);
        snprintf(err_, sizeof err_, "step: device fault code %u", fault);
        return -1;
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, d->ev0, d->ev1);
    stats.steps++;
    stats.tokens += n;
    int ns = 0;
    for (int i = 0; i < n; i++) ns += cols[i].sample ? 1 : 0;
    stats.sampled += ns;
    if (ns == n) { stats.decode_steps++; stats.decode_ms += ms; }
    stats.step_ms_last = ms;
    stats.step_ms_total += ms;
    stats.launches_per_step = d->launches;
    if (out_ids)
        for (int i = 0; i < n; i++) out_ids[i] = d->out_host[i];
    return 0;
}

}  // namespace cmolrt

namespace cmolrt {

// The GEMV launches of one single-column decode step, alone, replayed from a
// CUDA graph: every weight matrix of the model is streamed once per pass.
// The column is inactive (position -1), so no KV cache is written.
int Engine::gemv_sweep(int reps, double *ms_per_pass, long long *bytes_per_pass, int *launches_per_pass) {
    cudaSetDevice(device_);
    const int B = opt_.max_batch;
    int *m = d->meta_host;
    for (int i = 0; i < B; i++) { m[i] = 0; m[B + i] = -1; m[2 * B + i] = 0; m[3 * B + i] = 0; }
    m[4 * B] = 0;
    int launches = 0;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaMemcpyAsync(d->meta_dev, d->meta_host, d->meta_ints * sizeof(int), cudaMemcpyHostToDevice,
                                    d->stream);
    if (e == cudaSuccess) e = record_step(d, opt_, 1, max_pages_, launches, REC_MATMUL);   // eager warm-up
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        cudaError_t re = record_step(d, opt_, 1, max_pages_, launches, REC_MATMUL);
        e = cudaStreamEndCapture(d->stream, &g);
        if (re != cudaSuccess) e = re;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(ge, d->stream);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev0, d->stream);
    for (int r = 0; e == cudaSuccess && r < reps; r++) e = cudaGraphLaunch(ge, d->stream);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev1, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, d->ev0, d->ev1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        snprintf(err_, sizeof err_, "gemv_sweep: %s", cudaGetErrorString(e));
        return -1;
    }
    *ms_per_pass = (double)ms / reps;
    *bytes_per_pass = weight_bytes_;
    *launches_per_pass = launches;
    return 0;
}

int Engine::kernel_sweep(int what, int reps, double *ms_per_pass, long long *bytes_per_pass, double *flops_per_pass,
                         int *launches_per_pass) {
    if (last_n_ <= 0 || (what != 0 && what != 1) || reps <= 0) {
        snprintf(err_, sizeof err_, "kernel_sweep: no step has run yet, or bad arguments");
        return -1;
    }
    cudaSetDevice(device_);
    const int B = opt_.max_batch;
    int *m = d->meta_host;
    memcpy(m, last_meta_.data(), d->meta_ints * sizeof(int));
    m[4 * B] = 0;                                    // no page-table updates
    long long bytes = 0;
    double flops = 0.0;
    const HParams &hp = d->hp;
    if (what == 0) {
        for (int i = 0; i < B; i++) m[B + i] = -1;   // inactive: the products run, no KV is written
        bytes = weight_bytes_;
        flops = 2.0 * (double)weight_values_ * last_n_;
    } else {
        for (int i = 0; i < last_n_; i++) {
            const int pos = last_meta_[(size_t)B + i];
            if (pos < 0) continue;
            bytes += (long long)(pos + 1) * kv_bytes_per_token_;
            flops += 4.0 * hp.n_heads * hp.d_head * (pos + 1) * hp.n_layers;
        }
    }
    const int only = what == 0 ? REC_MATMUL : REC_ATTN;
    int launches = 0;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaMemcpyAsync(d->meta_dev, m, d->meta_ints * sizeof(int), cudaMemcpyHostToDevice, d->stream);
    if (e == cudaSuccess) e = record_step(d, opt_, last_bucket_, max_pages_, launches, only, last_grouped_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e == cudaSuccess) e = cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        cudaError_t re = record_step(d, opt_, last_bucket_, max_pages_, launches, only, last_grouped_);
        e = cudaStreamEndCapture(d->stream, &g);
        if (re != cudaSuccess) e = re;
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(ge, d->stream);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev0, d->stream);
    for (int r = 0; e == cudaSuccess && r < reps; r++) e = cudaGraphLaunch(ge, d->stream);
    if (e == cudaSuccess) e = cudaEventRecord(d->ev1, d->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, d->ev0, d->ev1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    // restore the last step's metadata on the device
    if (e == cudaSuccess) {
        memcpy(m, last_meta_.data(), d->meta_ints * sizeof(int));
        e = cudaMemcpyAsync(d->meta_dev, m, d->meta_ints * sizeof(int), cudaMemcpyHostToDevice, d->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    }
    if (e != cudaSuccess) {
        snprintf(err_, sizeof err_, "kernel_sweep: %s", cudaGetErrorString(e));
        return -1;
    }
    const unsigned int fault = fault_code();
    if (fault) {
        snprintf(err_, sizeof err_, "kernel_sweep: device fault code %u", fault);
        return -1;
    }
    *ms_per_pass = (double)ms / reps;
    *bytes_per_pass = bytes;
    *flops_per_pass = flops;
    *launches_per_pass = launches;
    return 0;
}

}  // namespace cmolrt
