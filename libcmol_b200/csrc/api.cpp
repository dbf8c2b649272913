// api.cpp — the libcmol public API (cmol.h, cmol_cuda.h) on the B200 engine.
//
// Structure:
//   cmol_model   — parsed GGUF (host), tokenizer, one Worker per GPU, the
//                  session slots and their pool lock;
//   Worker       — one scheduler thread per GPU that owns an Engine and runs
//                  the continuous batcher: every step packs all of its active
//                  requests (one token each: the next prompt token, or the
//                  last sampled token) into one decode step;
//   Request      — one cmol_generate_ids call; the caller thread blocks on it
//                  and runs the token callback, as src/api.c:494-500 of the
//                  reference does on its own thread.
//
// Generation semantics follow src/api.c:412-524: context-full check, prompt
// clamped to the free context, token-by-token prefill, RNG seeded once per
// call from params->seed, repeat window seeded with the prompt tail, then
// sample -> callback -> EOS stop -> window push -> max_new stop -> context
// stop -> forward.  A callback abort leaves the session's KV length where the
// reference would leave it (the aborted token is not part of it).
#include <errno.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "cmol.h"
#include "cmol_cuda.h"
#include "engine.h"
#include "host_model.h"
#include "tokenizer.h"

using namespace cmolrt;

namespace {

const int kRepeatBuf = 128;   // src/sampler.h:49

struct Request {
    cmol_session_t      *s = nullptr;
    std::vector<int32_t> prompt;
    cmol_gen_params_t    params = {};
    bool                 forward_only = false;   // teacher-forcing step, no sampling
    float               *logits_out = nullptr;
    // progress (worker thread only)
    int  start_n = 0;         // session n_tokens at admission
    long long budget = 0;     // tokens it may run (prompt + generation cap): its share of the GPU's load
    int  fed = 0;             // prompt tokens already run
    int  last = -1;           // sampled token waiting to be forwarded
    int  n_gen = 0;
    int  max_new = 0;
    bool admitted = false;
    // results (guarded by mu)
    std::mutex                            mu;
    std::condition_variable               cv;
    std::deque<std::pair<int32_t, int>>   q;       // (token, is_eos)
    bool                                  finished = false;
    cmol_err_t                            status = CMOL_OK;
    std::atomic<bool>                     abort{false};
    int                                   final_n_tokens = -1;
};

struct Worker;

}  // namespace

struct cmol_session {
    cmol_model_t *model = nullptr;
    int           slot = 0;           // index in the model's session table
    int           gpu = 0;
    int           lslot = 0;          // slot on its GPU's engine (page-table row, sampler state)
    int           n_tokens = 0;       // tokens in the KV cache
    std::vector<int> pages;            // page ids, one per page_tokens positions
};

namespace {

struct Worker {
    cmol_model_t          *m = nullptr;
    int                    index = 0;
    std::unique_ptr<Engine> eng;
    std::thread            th;
    std::mutex             mu;
    std::condition_variable cv;
    std::deque<Request *>  incoming;
    std::vector<Request *> active;
    std::vector<int>       free_pages;
    bool                   stop = false;
    int                    n_sessions = 0;     // sessions assigned (for placement)
    std::vector<int>       free_lslots;        // engine slots not held by a session
    // Placement load: tokens in the KV caches of this GPU's sessions plus
    // tokens still to run for their requests (prompt and generation budget).
    std::atomic<long long> load{0};
    void run();
};

}  // namespace

struct cmol_model {
    HostModel                 host;
    Tokenizer                 tok;
    cmol_config_t             cfg = {};
    std::vector<std::unique_ptr<Worker>> workers;
    std::vector<cmol_session> slots;
    std::vector<char>         slot_free;
    std::mutex                pool_mu;
    int                       eos = -1;
    int                       vocab = 0;
};

// ---------------------------------------------------------------------------
// configuration for the next cmol_load
// ---------------------------------------------------------------------------
static std::mutex g_cfg_mu;
static std::vector<int> g_devices;
static cmol_cuda_options_t g_opts = {0, 0.f, 0, 1, 0};

static void logf(const cmol_model_t *m, int level, const char *fmt, ...) {
    if (!m || !m->cfg.log_fn) return;
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    m->cfg.log_fn(level, buf, m->cfg.log_ud);
}

extern "C" cmol_err_t cmol_cuda_set_devices(const int *devices, int n) {
    if (n < 0 || (n > 0 && !devices)) return CMOL_ERR_ARGS;
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    g_devices.assign(devices, devices + n);
    return CMOL_OK;
}

extern "C" void cmol_cuda_set_options(const cmol_cuda_options_t *opt) {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (opt) g_opts = *opt;
    else g_opts = cmol_cuda_options_t{0, 0.f, 0, 1, 0};
}

static std::vector<int> pick_devices() {
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (!g_devices.empty()) return g_devices;
    std::vector<int> d;
    const char *env = getenv("CMOL_CUDA_DEVICES");
    if (env && *env) {
        const char *p = env;
        while (*p) {
            char *end = nullptr;
            long v = strtol(p, &end, 10);
            if (end == p) break;
            d.push_back((int)v);
            p = end;
            while (*p == ',' || *p == ' ') p++;
        }
    }
    if (d.empty()) d.push_back(0);
    return d;
}

// ---------------------------------------------------------------------------
// utilities (src/api.c:24-51)
// ---------------------------------------------------------------------------
extern "C" const char *cmol_strerror(cmol_err_t err) {
    switch (err) {
    case CMOL_OK: return "success";
    case CMOL_ERR_OOM: return "out of memory";
    case CMOL_ERR_IO: return "I/O error";
    case CMOL_ERR_INVALID: return "invalid or corrupt GGUF file";
    case CMOL_ERR_UNSUPPORTED: return "unsupported quantisation type or architecture";
    case CMOL_ERR_NO_SESSION: return "session pool exhausted \xe2\x80\x94 retry later";
    case CMOL_ERR_ARGS: return "invalid argument (NULL or out of range)";
    case CMOL_ERR_CTX_FULL: return "KV cache full \xe2\x80\x94 call cmol_session_reset()";
    case CMOL_ERR_TRUNC: return "output buffer too small (result truncated)";
    default: return "unknown error";
    }
}

extern "C" const char *cmol_version(void) { return CMOL_VERSION_STRING; }

// ---------------------------------------------------------------------------
// load / free
// ---------------------------------------------------------------------------
static void resolve_cfg(const HParams &hp, const cmol_config_t *in, cmol_config_t &c) {
    static const cmol_config_t def = CMOL_DEFAULT_CONFIG;
    c = in ? *in : def;
    if (c.max_ctx <= 0 || c.max_ctx > hp.model_max_ctx) c.max_ctx = hp.model_max_ctx;
    if (c.max_sessions <= 0) c.max_sessions = 4;
    if (c.prefill_chunk <= 0) c.prefill_chunk = 512;
}

extern "C" size_t cmol_arena_estimate(const char *path, const cmol_config_t *cfg) {
    if (!path) return 0;
    HParams hp;
    size_t nt = 0;
    if (gguf_peek(path, hp, nt) != CMOL_OK) return 0;
    cmol_config_t c;
    resolve_cfg(hp, cfg, c);
    const size_t kvd = (size_t)hp.n_kv_heads * (hp.n_heads ? hp.d_model / hp.n_heads : 0);
    // host: tensor table + tokenizer; device: KV (f32, full context) + activations
    size_t host = nt * sizeof(HTensor) + (size_t)hp.vocab_size * 80;
    size_t kv = 2 * (size_t)hp.n_layers * c.max_ctx * kvd * 4 * (size_t)c.max_sessions;
    size_t act = (size_t)c.max_sessions * 4 * (5 * (size_t)hp.d_model + 2 * (size_t)hp.d_ffn + hp.vocab_size);
    return sizeof(cmol_model) + host + kv + act;
}

extern "C" cmol_model_t *cmol_load(const char *path, const cmol_config_t *cfg, cmol_err_t *err) {
    if (!path) { if (err) *err = CMOL_ERR_ARGS; return nullptr; }
    HParams peek;
    size_t nt = 0;
    int rc = gguf_peek(path, peek, nt);
    if (rc) { if (err) *err = (cmol_err_t)rc; return nullptr; }
    cmol_model_t *m = new (std::nothrow) cmol_model();
    if (!m) { if (err) *err = CMOL_ERR_OOM; return nullptr; }
    resolve_cfg(peek, cfg, m->cfg);
    rc = gguf_load(path, m->host);
    if (rc) { delete m; if (err) *err = (cmol_err_t)rc; return nullptr; }
    rc = m->tok.build(m->host.vocab, m->host.hp.vocab_size);
    if (rc) { delete m; if (err) *err = (cmol_err_t)rc; return nullptr; }
    m->eos = m->host.vocab.eos;
    m->vocab = m->host.hp.vocab_size;

    const int ns = m->cfg.max_sessions;
    m->slots.resize((size_t)ns);
    m->slot_free.assign((size_t)ns, 1);
    for (int i = 0; i < ns; i++) { m->slots[i].model = m; m->slots[i].slot = i; }

    cmol_cuda_options_t opt;
    {
        std::lock_guard<std::mutex> lk(g_cfg_mu);
        opt = g_opts;
    }
    if (opt.kv_dtype != 0 && opt.kv_dtype != 1) {
        cmol_free(m);
        if (err) *err = CMOL_ERR_ARGS;
        return nullptr;
    }
    std::vector<int> devs = pick_devices();
    const int ng = (int)devs.size();
    std::vector<int> errs((size_t)ng, 0);
    std::vector<std::string> msgs((size_t)ng);
    m->workers.resize((size_t)ng);
    std::vector<std::thread> loaders;
    for (int g = 0; g < ng; g++) {
        m->workers[g].reset(new Worker());
        m->workers[g]->m = m;
        m->workers[g]->index = g;
        loaders.emplace_back([&, g]() {
            EngineOptions eo;
            const int per_gpu = (ns + ng - 1) / ng;
            eo.max_slots = per_gpu;          // this GPU's share of the sessions
            // columns of a step: one per session, plus up to prefill_chunk
            // (at most 256) further prompt tokens of sessions still in prefill
            const int prefill = std::max(1, std::min(m->cfg.prefill_chunk, 256));
            eo.max_batch = (opt.max_batch > 0 ? std::min(opt.max_batch, per_gpu) : per_gpu) + (prefill > 1 ? prefill : 0);
            eo.max_group = prefill;
            eo.max_ctx = m->cfg.max_ctx;
            eo.page_tokens = opt.kv_page_tokens > 0 ? opt.kv_page_tokens : 64;
            eo.kv_pool_frac = opt.kv_pool_frac > 0.f ? opt.kv_pool_frac : 0.85f;
            eo.use_graphs = opt.use_graphs != 0;
            eo.kv_f16 = opt.kv_dtype == 1;
            eo.split_tokens = 64;
            if (eo.split_tokens % eo.page_tokens) eo.split_tokens = eo.page_tokens * 4;
            char msg[256] = {0};
            int e = 0;
            Engine *en = Engine::create(devs[g], m->host, eo, &e, msg, sizeof msg);
            errs[g] = e;
            msgs[g] = msg;
            if (en) {
                m->workers[g]->eng.reset(en);
                // pages per GPU: the pool is shared by that GPU's sessions
                std::vector<int> &fp = m->workers[g]->free_pages;
                fp.resize((size_t)en->n_pages());
                for (int i = 0; i < en->n_pages(); i++) fp[i] = en->n_pages() - 1 - i;
                std::vector<int> &fl = m->workers[g]->free_lslots;
                for (int i = per_gpu - 1; i >= 0; i--) fl.push_back(i);
            }
        });
    }
    for (auto &t : loaders) t.join();
    for (int g = 0; g < ng; g++) {
        if (errs[g]) {
            logf(m, CMOL_LOG_ERROR, "cmol_load: GPU %d: %s", devs[g], msgs[g].c_str());
            cmol_err_t e = (cmol_err_t)errs[g];
            cmol_free(m);
            if (err) *err = e;
            return nullptr;
        }
    }
    for (auto &w : m->workers) w->th = std::thread([wp = w.get()]() { wp->run(); });
    const HParams &hp = m->host.hp;
    logf(m, CMOL_LOG_INFO,
         "cmol_load: arch=%s layers=%d heads=%d/%d d=%d ffn=%d vocab=%d ctx=%d sessions=%d kernel=cuda-sm100a gpus=%d",
         hp.arch.c_str(), hp.n_layers, hp.n_heads, hp.n_kv_heads, hp.d_model, hp.d_ffn, hp.vocab_size,
         m->cfg.max_ctx, ns, ng);
    if (err) *err = CMOL_OK;
    return m;
}

extern "C" void cmol_free(cmol_model_t *m) {
    if (!m) return;
    for (auto &w : m->workers) {
        if (!w) continue;
        {
            std::lock_guard<std::mutex> lk(w->mu);
            w->stop = true;
        }
        w->cv.notify_all();
        if (w->th.joinable()) w->th.join();
        w->eng.reset();
    }
    delete m;
}

// ---------------------------------------------------------------------------
// sessions (src/api.c:309-334): lowest free slot, NULL when exhausted
// ---------------------------------------------------------------------------
// Placement (scope of the survey's multi-GPU row): a new session goes to
// the GPU with the least outstanding work — tokens held in its sessions' KV
// caches plus tokens its queued and running requests still have to run —
// among those with a free engine slot; ties go to the GPU with fewer
// sessions, then the lower index.
extern "C" cmol_session_t *cmol_session_acquire(cmol_model_t *m) {
    if (!m) return nullptr;
    std::lock_guard<std::mutex> lk(m->pool_mu);
    for (size_t i = 0; i < m->slot_free.size(); i++) {
        if (!m->slot_free[i]) continue;
        int best = -1;
        for (size_t g = 0; g < m->workers.size(); g++) {
            Worker *w = m->workers[g].get();
            if (w->free_lslots.empty()) continue;
            if (best < 0) { best = (int)g; continue; }
            Worker *b = m->workers[(size_t)best].get();
            const long long lw = w->load.load(), lb = b->load.load();
            if (lw < lb || (lw == lb && w->n_sessions < b->n_sessions)) best = (int)g;
        }
        if (best < 0) return nullptr;   // every engine slot is held
        m->slot_free[i] = 0;
        cmol_session_t *s = &m->slots[i];
        Worker *w = m->workers[(size_t)best].get();
        s->gpu = best;
        s->lslot = w->free_lslots.back();
        w->free_lslots.pop_back();
        w->n_sessions++;
        s->n_tokens = 0;
        return s;
    }
    return nullptr;
}

extern "C" void cmol_session_release(cmol_session_t *s) {
    if (!s) return;
    cmol_model_t *m = s->model;
    Worker *w = m->workers[(size_t)s->gpu].get();
    {
        std::lock_guard<std::mutex> lk(w->mu);
        for (int p : s->pages) w->free_pages.push_back(p);
    }
    s->pages.clear();
    w->load -= s->n_tokens;
    s->n_tokens = 0;
    std::lock_guard<std::mutex> lk(m->pool_mu);
    w->n_sessions--;
    w->free_lslots.push_back(s->lslot);
    m->slot_free[(size_t)s->slot] = 1;
}

extern "C" void cmol_session_reset(cmol_session_t *s) {
    if (!s) return;
    s->model->workers[(size_t)s->gpu]->load -= s->n_tokens;
    s->n_tokens = 0;   // pages stay with the session for its next turn
}

// ---------------------------------------------------------------------------
// Session KV snapshots: a header and the K / V of every page the session's
// context occupies, all layers, in the engine's KV format.
// ---------------------------------------------------------------------------
namespace {
struct KvSnapshotHeader {
    uint32_t magic, version;
    int32_t  n_layers, page_tokens, kv_f16, vocab;
    int64_t  page_bytes;                 // one page of one layer
    int32_t  n_tokens, n_pages;
};
const uint32_t kSnapMagic = 0x564B4D43u;   // "CMKV"
}  // namespace

extern "C" cmol_err_t cmol_cuda_session_save(cmol_session_t *s, void *buf, size_t cap, size_t *size) {
    if (!s || !size) return CMOL_ERR_ARGS;
    Engine *e = s->model->workers[(size_t)s->gpu]->eng.get();
    const int P = e->page_tokens();
    KvSnapshotHeader h = {};
    h.magic = kSnapMagic;
    h.version = 1;
    h.n_layers = e->n_layers();
    h.page_tokens = P;
    h.kv_f16 = e->kv_f16() ? 1 : 0;
    h.vocab = s->model->vocab;
    h.page_bytes = e->kv_page_bytes();
    h.n_tokens = s->n_tokens;
    h.n_pages = (s->n_tokens + P - 1) / P;
    const size_t need = sizeof h + (size_t)h.n_layers * h.n_pages * (size_t)h.page_bytes;
    *size = need;
    if (!buf) return CMOL_OK;
    if (cap < need) return CMOL_ERR_TRUNC;
    if (h.n_pages > (int)s->pages.size()) return CMOL_ERR_INVALID;
    memcpy(buf, &h, sizeof h);
    if (e->kv_pages_copy(s->pages.data(), h.n_pages, static_cast<unsigned char *>(buf) + sizeof h, true) != 0)
        return CMOL_ERR_INVALID;
    return CMOL_OK;
}

extern "C" cmol_err_t cmol_cuda_session_restore(cmol_session_t *s, const void *buf, size_t size) {
    if (!s || !buf || size < sizeof(KvSnapshotHeader)) return CMOL_ERR_ARGS;
    KvSnapshotHeader h;
    memcpy(&h, buf, sizeof h);
    Worker *w = s->model->workers[(size_t)s->gpu].get();
    Engine *e = w->eng.get();
    const int P = e->page_tokens();
    if (h.magic != kSnapMagic || h.version != 1 || h.n_layers != e->n_layers() || h.page_tokens != P ||
        h.kv_f16 != (e->kv_f16() ? 1 : 0) || h.vocab != s->model->vocab || h.page_bytes != e->kv_page_bytes() ||
        h.n_tokens < 0 || h.n_pages != (h.n_tokens + P - 1) / P)
        return CMOL_ERR_INVALID;
    if (h.n_tokens > e->max_ctx()) return CMOL_ERR_CTX_FULL;
    if (size != sizeof h + (size_t)h.n_layers * h.n_pages * (size_t)h.page_bytes) return CMOL_ERR_ARGS;
    {
        // the session's own pages first, then pages from its GPU's free list
        std::lock_guard<std::mutex> lk(w->mu);
        const size_t want = (size_t)h.n_pages;
        if (s->pages.size() < want && w->free_pages.size() < want - s->pages.size()) return CMOL_ERR_OOM;
        while (s->pages.size() < want) {
            s->pages.push_back(w->free_pages.back());
            w->free_pages.pop_back();
        }
    }
    if (e->kv_pages_copy(s->pages.data(), h.n_pages, const_cast<unsigned char *>(
                                                          static_cast<const unsigned char *>(buf) + sizeof h),
                         false) != 0 ||
        e->set_page_row(s->lslot, s->pages.data(), (int)s->pages.size()) != 0)
        return CMOL_ERR_INVALID;
    w->load += h.n_tokens - s->n_tokens;
    s->n_tokens = h.n_tokens;
    return CMOL_OK;
}

extern "C" int cmol_session_n_tokens(const cmol_session_t *s) { return s ? s->n_tokens : 0; }
extern "C" int cmol_session_device(const cmol_session_t *s) { return s ? s->gpu : -1; }
extern "C" int cmol_vocab_size(const cmol_model_t *m) { return m ? m->vocab : 0; }
extern "C" int cmol_eos_id(const cmol_model_t *m) { return m ? m->eos : -1; }
extern "C" int cmol_cuda_n_gpus(const cmol_model_t *m) { return m ? (int)m->workers.size() : 0; }

// ---------------------------------------------------------------------------
// tokenizer + ChatML (src/api.c:340-398)
// ---------------------------------------------------------------------------
extern "C" int cmol_encode(cmol_model_t *m, const char *text, int32_t *out, int out_cap) {
    if (!m || !text || !out || out_cap <= 0) return CMOL_ERR_ARGS;
    return m->tok.encode(text, out, out_cap, m->tok.add_bos());
}

extern "C" const char *cmol_decode_token(cmol_model_t *m, int32_t id) {
    if (!m) return nullptr;
    return m->tok.decode(id);
}

extern "C" int cmol_format_chatml(const char *system, const char *user, char *buf, size_t cap) {
    if (!user) return CMOL_ERR_ARGS;
    const char *sys = system ? system : "";
    int n;
    if (sys[0])
        n = snprintf(buf, cap, "<|im_start|>system\n%s<|im_end|>\n<|im_start|>user\n%s<|im_end|>\n<|im_start|>assistant\n",
                     sys, user);
    else
        n = snprintf(buf, cap, "<|im_start|>user\n%s<|im_end|>\n<|im_start|>assistant\n", user);
    if (n < 0) return CMOL_ERR_ARGS;
    if (buf && cap > 0 && (size_t)n >= cap) return CMOL_ERR_TRUNC;
    return n;
}

extern "C" int cmol_format_chatml_turn(const char *user, char *buf, size_t cap) {
    if (!user) return CMOL_ERR_ARGS;
    int n = snprintf(buf, cap, "<|im_end|>\n<|im_start|>user\n%s<|im_end|>\n<|im_start|>assistant\n", user);
    if (n < 0) return CMOL_ERR_ARGS;
    if (buf && cap > 0 && (size_t)n >= cap) return CMOL_ERR_TRUNC;
    return n;
}

// ---------------------------------------------------------------------------
// the batcher
// ---------------------------------------------------------------------------
namespace {

// splitmix64 expansion of a 32-bit seed into xoshiro256** state; seed 0 =
// time-based (src/sampler.c:52-75).
uint64_t splitmix(uint64_t *x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

void seed_rng(uint64_t st[4], unsigned seed, const void *salt) {
    uint64_t x;
    if (seed == 0) {
        static std::atomic<uint64_t> ctr{0};
        x = (uint64_t)time(nullptr);
        x ^= (++ctr) * 6364136223846793005ULL;
        x ^= (uint64_t)(uintptr_t)salt;
        if (!x) x = 0xDEADBEEFCAFEBABEULL;
    } else {
        x = (uint64_t)seed;
    }
    for (int i = 0; i < 4; i++) st[i] = splitmix(&x);
}

void finish(Request *r, cmol_err_t st) {
    std::lock_guard<std::mutex> lk(r->mu);
    r->status = st;
    r->finished = true;
    r->cv.notify_all();
}

void Worker::run() {
    Engine *e = eng.get();
    std::vector<StepColumn> cols;
    std::vector<PageUpdate> upd;
    std::vector<Request *> batch;
    std::vector<int32_t> out;
    std::vector<float> logits;      // [columns][vocab] of a teacher-forcing step
    const int P = e->page_tokens();
    // A request belongs to the thread waiting in submit_and_wait, which may
    // return (and destroy it) as soon as finish() signals it: so a request is
    // first retired (session pointer cleared, status queued), then removed
    // from `active`, and only then finished, as the worker's last touch.
    std::vector<std::pair<Request *, cmol_err_t>> retired;
    auto retire = [&](Request *r, cmol_err_t st) {
        load -= r->budget - (r->s->n_tokens - r->start_n);   // what it did not run leaves the load
        r->s = nullptr;
        retired.emplace_back(r, st);
    };
    for (;;) {
        if (!retired.empty()) {
            active.erase(std::remove_if(active.begin(), active.end(), [](Request *r) { return r->s == nullptr; }),
                         active.end());
            for (auto &rs : retired) finish(rs.first, rs.second);
            retired.clear();
        }
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return stop || !incoming.empty() || !active.empty(); });
            if (stop && incoming.empty() && active.empty()) return;
            while (!incoming.empty()) {
                active.push_back(incoming.front());
                incoming.pop_front();
            }
        }
        // admit new requests: sampler state
        for (Request *r : active) {
            if (r->admitted) continue;
            r->admitted = true;
            if (r->forward_only) continue;
            SamplerParams sp;
            sp.temperature = r->params.temperature;
            sp.top_p = r->params.top_p;
            sp.top_k = r->params.top_k;
            sp.repeat_penalty = r->params.repeat_penalty;
            sp.eos = m->eos;
            seed_rng((uint64_t *)sp.rng, r->params.seed, r);
            int last_n = r->params.repeat_last_n;
            if (last_n <= 0 || last_n > kRepeatBuf) last_n = kRepeatBuf;
            const int np = (int)r->prompt.size();
            const int seed_n = np < last_n ? np : last_n;
            for (int i = 0; i < seed_n; i++) sp.ring[i] = r->prompt[(size_t)(np - seed_n + i)];
            sp.ring_head = seed_n % kRepeatBuf;
            sp.ring_fill = seed_n;
            if (e->set_sampler(r->s->lslot, sp)) retire(r, CMOL_ERR_INVALID);
        }
        // drop aborted / failed requests
        std::vector<Request *> keep;
        for (Request *r : active) {
            if (!r->s) continue;
            if (r->abort.load()) {
                r->s->n_tokens = r->final_n_tokens >= 0 ? r->final_n_tokens : r->s->n_tokens;
                load -= r->budget - (r->s->n_tokens - r->start_n);
                finish(r, CMOL_OK);
                continue;
            }
            keep.push_back(r);
        }
        active.swap(keep);
        if (active.empty()) continue;

        // build the step: forward-only (teacher-forcing) requests run
        // together, in a step of their own
        cols.clear();
        upd.clear();
        batch.clear();
        bool fwd = false;
        for (Request *r : active)
            if (r->forward_only) { fwd = true; break; }
        const int cap = e->max_batch();
        const int prefill = std::max(1, std::min(m->cfg.prefill_chunk, 256));
        struct Entry {
            Request *r;
            int n;        // columns of this request in the step
            int scol;     // the column whose sampled token it takes, or -1
            int c0;       // its first column
        };
        std::vector<Entry> ent;
        // one column of request r at offset `off` past its next token; false
        // when no KV page is left for it
        auto add_col = [&](Request *r, int off) -> bool {
            cmol_session_t *s = r->s;
            StepColumn c;
            c.pos = s->n_tokens + off;
            c.slot = s->lslot;
            const int np = (int)r->prompt.size();
            if (r->fed + off < np) {
                c.token = r->prompt[(size_t)(r->fed + off)];
                c.sample = (!r->forward_only && r->fed + off == np - 1) ? 1 : 0;
            } else {
                c.token = r->last;
                c.sample = 1;
            }
            const int pidx = c.pos / P;
            if (pidx >= (int)s->pages.size()) {
                std::lock_guard<std::mutex> lk(mu);
                if (free_pages.empty()) return false;
                int pg = free_pages.back();
                free_pages.pop_back();
                s->pages.push_back(pg);
                upd.push_back(PageUpdate{s->lslot, pidx, pg});
            }
            cols.push_back(c);
            return true;
        };
        // pass 1: the next token of every request (decode or prompt);
        // pass 2: batched prefill, further prompt tokens of the same sessions as
        // columns at consecutive positions (each step's Q/K/V kernel writes all
        // columns' keys and values before attention reads them, so a column
        // attends to the prompt tokens before it in the same step).  A session's
        // columns are emitted together, in increasing position: attention serves
        // such a group from one load of its keys and values.
        std::vector<int> want;
        std::vector<Request *> order;
        int ncols = 0;
        for (Request *r : active) {
            if (fwd && !r->forward_only) continue;
            if (ncols >= cap) break;
            order.push_back(r);
            want.push_back(1);
            ncols++;
        }
        if (!fwd && prefill > 1) {
            for (size_t i = 0; i < order.size() && ncols < cap; i++) {
                Request *r = order[i];
                const int np = (int)r->prompt.size();
                while (want[i] < prefill && r->fed + want[i] < np && ncols < cap) {
                    want[i]++;
                    ncols++;
                }
            }
        }
        for (size_t i = 0; i < order.size(); i++) {
            Request *r = order[i];
            Entry en{r, 0, -1, (int)cols.size()};
            for (int k = 0; k < want[i]; k++) {
                if (!add_col(r, k)) break;          // no KV page left: take fewer tokens
                if (cols.back().sample) en.scol = (int)cols.size() - 1;
                en.n++;
            }
            if (en.n == 0) { retire(r, CMOL_ERR_OOM); continue; }
            ent.push_back(en);
            batch.push_back(r);
        }
        if (batch.empty()) continue;
        out.assign(cols.size(), -1);
        float *lg = nullptr;
        if (fwd) {
            logits.resize(cols.size() * (size_t)m->vocab);
            lg = logits.data();
        }
        if (e->step(cols, upd, out.data(), lg) != 0) {
            logf(m, CMOL_LOG_ERROR, "decode step failed on GPU %d: %s", e->device(), e->last_error());
            for (Request *r : batch) retire(r, CMOL_ERR_INVALID);
            continue;
        }
        // advance every request of the step
        for (const Entry &en : ent) {
            Request *r = en.r;
            cmol_session_t *s = r->s;
            s->n_tokens += en.n;
            const int np = (int)r->prompt.size();
            if (r->fed < np) r->fed += en.n;
            if (r->forward_only) {
                memcpy(r->logits_out, lg + (size_t)en.c0 * m->vocab, (size_t)m->vocab * sizeof(float));
                retire(r, CMOL_OK);
                continue;
            }
            if (en.scol < 0) continue;
            const int32_t t = out[(size_t)en.scol];
            const int is_eos = (m->eos >= 0 && t == m->eos) ? 1 : 0;
            bool done = false;
            if (is_eos) {
                done = true;
            } else {
                r->n_gen++;
                if (r->max_new > 0 && r->n_gen >= r->max_new) done = true;       // src/api.c:509-510
                else if (s->n_tokens >= m->cfg.max_ctx) done = true;            // src/api.c:513
                else r->last = t;
            }
            {
                std::lock_guard<std::mutex> lk(r->mu);
                r->q.emplace_back(t, is_eos);
                r->cv.notify_all();
            }
            if (done) retire(r, CMOL_OK);
        }
        keep.clear();
        for (Request *r : active)
            if (r->s) keep.push_back(r);
        active.swap(keep);
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// generation entry points
// ---------------------------------------------------------------------------
static cmol_err_t submit_and_wait(cmol_session_t *s, Request &r, cmol_id_cb_t cb_id, cmol_token_cb_t cb_txt,
                                  void *ud) {
    cmol_model_t *m = s->model;
    Worker *w = m->workers[(size_t)s->gpu].get();
    r.s = s;
    r.start_n = s->n_tokens;
    w->load += r.budget;
    {
        std::lock_guard<std::mutex> lk(w->mu);
        w->incoming.push_back(&r);
    }
    w->cv.notify_all();
    int consumed = 0;
    bool aborted = false;
    for (;;) {
        std::pair<int32_t, int> item;
        {
            std::unique_lock<std::mutex> lk(r.mu);
            r.cv.wait(lk, [&] { return r.finished || !r.q.empty(); });
            if (r.q.empty()) break;               // finished and drained
            item = r.q.front();
            r.q.pop_front();
        }
        if (aborted) continue;
        int stop = 0;
        if (cb_id) stop = cb_id(item.first, item.second, ud);
        if (cb_txt) {
            const char *piece = m->tok.decode(item.first);
            stop = cb_txt(piece ? piece : "", piece ? strlen(piece) : 0, item.second, ud);
        }
        consumed++;
        if (stop && !item.second) {
            // the reference stops before forwarding this token (src/api.c:498-499)
            {
                std::lock_guard<std::mutex> lk(r.mu);
                r.final_n_tokens = r.start_n + (int)r.prompt.size() + consumed - 1;
            }
            r.abort.store(true);
            w->cv.notify_all();
            aborted = true;
        }
    }
    // the worker no longer touches the session once the request finished
    if (aborted) s->n_tokens = r.final_n_tokens;
    return r.status;
}

// The checks and set-up of one generation request (src/api.c:420-436):
// context-full check, prompt clamped to the free context, token ids in
// range.  *empty: nothing to run (an empty prompt), the call returns OK.
static cmol_err_t prepare_request(cmol_session_t *s, const int32_t *prompt, int n_prompt,
                                  const cmol_gen_params_t *params, Request &r, bool *empty) {
    static const cmol_gen_params_t def = CMOL_DEFAULT_PARAMS;
    *empty = false;
    if (!s || (!prompt && n_prompt > 0) || n_prompt < 0) return CMOL_ERR_ARGS;
    if (!params) params = &def;
    cmol_model_t *m = s->model;
    if (s->n_tokens >= m->cfg.max_ctx) return CMOL_ERR_CTX_FULL;   // src/api.c:426
    if (n_prompt == 0) { *empty = true; return CMOL_OK; }
    const int avail = m->cfg.max_ctx - s->n_tokens;
    if (n_prompt > avail) n_prompt = avail;
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->vocab) return CMOL_ERR_ARGS;
    r.prompt.assign(prompt, prompt + n_prompt);
    r.params = *params;
    r.max_new = params->max_new_tokens < 0 ? m->cfg.max_ctx : params->max_new_tokens;
    r.budget = std::min<long long>((long long)n_prompt + r.max_new, m->cfg.max_ctx - s->n_tokens);
    return CMOL_OK;
}

static cmol_err_t generate_ids_impl(cmol_session_t *s, const int32_t *prompt, int n_prompt,
                                    const cmol_gen_params_t *params, cmol_id_cb_t cb_id, cmol_token_cb_t cb_txt,
                                    void *ud) {
    Request r;
    bool empty = false;
    const cmol_err_t st = prepare_request(s, prompt, n_prompt, params, r, &empty);
    if (st != CMOL_OK || empty) return st;
    return submit_and_wait(s, r, cb_id, cb_txt, ud);
}

extern "C" cmol_err_t cmol_generate_ids(cmol_session_t *s, const int32_t *prompt, int n_prompt,
                                        const cmol_gen_params_t *params, cmol_id_cb_t on_token, void *ud) {
    return generate_ids_impl(s, prompt, n_prompt, params, on_token, nullptr, ud);
}

extern "C" cmol_err_t cmol_generate(cmol_session_t *s, const char *prompt, const cmol_gen_params_t *params,
                                    cmol_token_cb_t on_token, void *ud) {
    if (!s || !prompt) return CMOL_ERR_ARGS;
    cmol_model_t *m = s->model;
    if (s->n_tokens >= m->cfg.max_ctx) return CMOL_ERR_CTX_FULL;
    std::vector<int32_t> ids((size_t)m->cfg.max_ctx);
    int n = m->tok.encode(prompt, ids.data(), m->cfg.max_ctx, m->tok.add_bos());
    if (n < 0) return (cmol_err_t)n;
    if (n == 0) return CMOL_OK;
    return generate_ids_impl(s, ids.data(), n, params, nullptr, on_token, ud);
}

extern "C" cmol_err_t cmol_forward_logits(cmol_session_t *s, int32_t token, float *logits_out) {
    if (!s || !logits_out) return CMOL_ERR_ARGS;
    cmol_model_t *m = s->model;
    if (token < 0 || token >= m->vocab) return CMOL_ERR_ARGS;
    if (s->n_tokens >= m->cfg.max_ctx) return CMOL_ERR_CTX_FULL;
    Request r;
    r.prompt.assign(1, token);
    r.forward_only = true;
    r.logits_out = logits_out;
    r.budget = 1;
    return submit_and_wait(s, r, nullptr, nullptr, nullptr);
}

extern "C" cmol_err_t cmol_forward_logits_batch(cmol_session_t *const *ss, const int32_t *tokens, int n,
                                                float *logits_out) {
    if (!ss || !tokens || !logits_out || n <= 0 || !ss[0]) return CMOL_ERR_ARGS;
    cmol_model_t *m = ss[0]->model;
    const int gpu = ss[0]->gpu;
    Worker *w = m->workers[(size_t)gpu].get();
    if (n > w->eng->max_batch()) return CMOL_ERR_ARGS;
    for (int i = 0; i < n; i++) {
        if (!ss[i] || ss[i]->model != m || ss[i]->gpu != gpu) return CMOL_ERR_ARGS;
        if (tokens[i] < 0 || tokens[i] >= m->vocab) return CMOL_ERR_ARGS;
        if (ss[i]->n_tokens >= m->cfg.max_ctx) return CMOL_ERR_CTX_FULL;
        for (int j = 0; j < i; j++)
            if (ss[j] == ss[i]) return CMOL_ERR_ARGS;
    }
    std::vector<std::unique_ptr<Request>> rs;
    rs.reserve((size_t)n);
    for (int i = 0; i < n; i++) {
        rs.emplace_back(new Request());
        Request &r = *rs.back();
        r.s = ss[i];
        r.start_n = ss[i]->n_tokens;
        r.prompt.assign(1, tokens[i]);
        r.forward_only = true;
        r.logits_out = logits_out + (size_t)i * m->vocab;
        r.budget = 1;
    }
    {
        // one hand-over: the worker takes all of them into the same step
        std::lock_guard<std::mutex> lk(w->mu);
        for (auto &r : rs) {
            w->load += r->budget;
            w->incoming.push_back(r.get());
        }
    }
    w->cv.notify_all();
    cmol_err_t st = CMOL_OK;
    for (auto &r : rs) {
        std::unique_lock<std::mutex> lk(r->mu);
        r->cv.wait(lk, [&] { return r->finished; });
        if (r->status != CMOL_OK && st == CMOL_OK) st = r->status;
    }
    return st;
}

extern "C" cmol_err_t cmol_generate_batch(cmol_batch_item_t *items, int n) {
    if (!items || n <= 0) return CMOL_ERR_ARGS;
    // every request is set up first and handed to its GPU's batcher in one
    // go, so the first step already holds all of them; tokens are collected
    // when a request has finished (no callback runs)
    std::vector<std::unique_ptr<Request>> rs((size_t)n);
    for (int i = 0; i < n; i++) {
        cmol_batch_item_t &it = items[i];
        it.n_out = 0;
        std::unique_ptr<Request> r(new Request());
        bool empty = false;
        it.status = prepare_request(it.session, it.prompt, it.n_prompt, it.params, *r, &empty);
        if (it.status != CMOL_OK || empty) continue;
        r->s = it.session;
        r->start_n = it.session->n_tokens;
        rs[(size_t)i] = std::move(r);
    }
    std::vector<Worker *> touched;
    for (int i = 0; i < n; i++) {
        if (!rs[(size_t)i]) continue;
        cmol_session_t *s = items[i].session;
        Worker *w = s->model->workers[(size_t)s->gpu].get();
        if (std::find(touched.begin(), touched.end(), w) == touched.end()) touched.push_back(w);
    }
    for (Worker *w : touched) {
        {
            std::lock_guard<std::mutex> lk(w->mu);
            for (int i = 0; i < n; i++) {
                if (!rs[(size_t)i]) continue;
                cmol_session_t *s = items[i].session;
                if (s->model->workers[(size_t)s->gpu].get() == w) {
                    w->load += rs[(size_t)i]->budget;
                    w->incoming.push_back(rs[(size_t)i].get());
                }
            }
        }
        w->cv.notify_all();
    }
    for (int i = 0; i < n; i++) {
        Request *r = rs[(size_t)i].get();
        if (!r) continue;
        std::unique_lock<std::mutex> lk(r->mu);
        r->cv.wait(lk, [&] { return r->finished; });
        cmol_batch_item_t &it = items[i];
        for (const auto &tk : r->q) {
            if (it.n_out < it.out_cap) it.out[it.n_out] = tk.first;
            it.n_out++;
        }
        if (it.n_out > it.out_cap) it.n_out = it.out_cap;
        it.status = r->status;
    }
    for (int i = 0; i < n; i++)
        if (items[i].status != CMOL_OK) return items[i].status;
    return CMOL_OK;
}

// ---------------------------------------------------------------------------
// measurement
// ---------------------------------------------------------------------------
extern "C" cmol_err_t cmol_cuda_stats(const cmol_model_t *m, int g, cmol_cuda_stats_t *out) {
    if (!m || !out || g < 0 || g >= (int)m->workers.size()) return CMOL_ERR_ARGS;
    const Engine *e = m->workers[(size_t)g]->eng.get();
    memset(out, 0, sizeof *out);
    out->decode_steps = e->stats.decode_steps;
    out->decode_tokens = e->stats.sampled;
    out->prefill_tokens = e->stats.tokens - e->stats.sampled;
    out->decode_ms = e->stats.decode_ms;
    out->step_ms_last = e->stats.step_ms_last;
    out->weight_bytes = e->weight_bytes_per_step();
    out->kernel_launches_per_step = e->stats.launches_per_step;
    out->graph_steps = (int)e->stats.graph_steps;
    out->steps = e->stats.steps;
    out->step_ms_total = e->stats.step_ms_total;
    out->last_fault_code = e->last_fault();
    out->h2d_bytes_per_step = e->h2d_bytes_per_step();
    out->d2h_bytes_per_step = e->d2h_bytes_per_step();
    return CMOL_OK;
}

extern "C" cmol_err_t cmol_cuda_kernel_sweep(cmol_model_t *m, int g, int what, int reps, double *ms_per_pass,
                                             long long *bytes_per_pass, double *flops_per_pass,
                                             int *launches_per_pass) {
    if (!m || g < 0 || g >= (int)m->workers.size() || reps <= 0 || !ms_per_pass || !bytes_per_pass ||
        !flops_per_pass || !launches_per_pass)
        return CMOL_ERR_ARGS;
    Worker *w = m->workers[(size_t)g].get();
    std::lock_guard<std::mutex> lk(w->mu);
    if (!w->active.empty() || !w->incoming.empty()) return CMOL_ERR_NO_SESSION;
    if (w->eng->kernel_sweep(what, reps, ms_per_pass, bytes_per_pass, flops_per_pass, launches_per_pass)) {
        logf(m, CMOL_LOG_ERROR, "%s", w->eng->last_error());
        return CMOL_ERR_INVALID;
    }
    return CMOL_OK;
}

extern "C" cmol_err_t cmol_cuda_debug_inject(cmol_model_t *m, int g, int kind) {
    if (!m || g < 0 || g >= (int)m->workers.size() || kind < 1 || kind > 3) return CMOL_ERR_ARGS;
    m->workers[(size_t)g]->eng->inject_fault(kind);
    return CMOL_OK;
}

extern "C" void cmol_cuda_stats_reset(cmol_model_t *m) {
    if (!m) return;
    for (auto &w : m->workers) w->eng->reset_stats();
}

// ---------------------------------------------------------------------------
// host-only tokenizer handle (cmolcu.h): the GGUF vocabulary without loading
// weights or touching a GPU
// ---------------------------------------------------------------------------
struct cmolcu_tokenizer {
    HostModel host;
    Tokenizer tok;
};

extern "C" int cmolcu_tokenizer_open(const char *path, cmolcu_tokenizer **out) {
    if (!path || !out) return CMOL_ERR_ARGS;
    *out = nullptr;
    cmolcu_tokenizer *t = new (std::nothrow) cmolcu_tokenizer();
    if (!t) return CMOL_ERR_OOM;
    int rc = gguf_load(path, t->host);
    if (!rc) rc = t->tok.build(t->host.vocab, t->host.hp.vocab_size);
    if (rc) { delete t; return rc; }
    *out = t;
    return CMOL_OK;
}

extern "C" int cmolcu_tokenizer_encode(const cmolcu_tokenizer *t, const char *text, int32_t *out, int cap) {
    if (!t) return CMOL_ERR_ARGS;
    return t->tok.encode(text, out, cap, t->tok.add_bos());
}

extern "C" const char *cmolcu_tokenizer_decode(const cmolcu_tokenizer *t, int32_t id) {
    return t ? t->tok.decode(id) : nullptr;
}

extern "C" void cmolcu_tokenizer_free(cmolcu_tokenizer *t) { delete t; }

extern "C" cmol_err_t cmol_cuda_gemv_sweep(cmol_model_t *m, int g, int reps, double *ms_per_pass,
                                          long long *bytes_per_pass, int *launches_per_pass) {
    if (!m || g < 0 || g >= (int)m->workers.size() || reps <= 0 || !ms_per_pass || !bytes_per_pass ||
        !launches_per_pass)
        return CMOL_ERR_ARGS;
    Worker *w = m->workers[(size_t)g].get();
    // run on the worker's engine while no request is active on it
    std::lock_guard<std::mutex> lk(w->mu);
    if (!w->active.empty() || !w->incoming.empty()) return CMOL_ERR_NO_SESSION;
    if (w->eng->gemv_sweep(reps, ms_per_pass, bytes_per_pass, launches_per_pass)) {
        logf(m, CMOL_LOG_ERROR, "%s", w->eng->last_error());
        return CMOL_ERR_INVALID;
    }
    return CMOL_OK;
}
