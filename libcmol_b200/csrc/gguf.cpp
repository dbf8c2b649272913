// gguf.cpp — GGUF v2/v3 reader for the host runtime (see host_model.h).
#include "host_model.h"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "cmol.h"

namespace cmolrt {

namespace {

enum : uint32_t {
    T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64
};

int scalar_width(uint32_t t) {
    static const int w[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    return t < 13 ? w[t] : -1;
}

// Bounds-checked cursor; once `bad` is set every read yields zero.
struct Reader {
    const uint8_t *p;
    size_t         n, off = 0;
    bool           bad = false;

    bool need(size_t k) {
        if (bad || k > n - off) { bad = true; return false; }
        return true;
    }
    template <typename T> T get() {
        T v{};
        if (need(sizeof(T))) { memcpy(&v, p + off, sizeof(T)); off += sizeof(T); }
        return v;
    }
    std::string str() {
        uint64_t len = get<uint64_t>();
        if (len > ((uint64_t)128 << 20) || !need((size_t)len)) { bad = true; return {}; }
        std::string s((const char *)p + off, (size_t)len);
        off += (size_t)len;
        return s;
    }
    void skip_scalar(uint32_t t) {
        if (t == T_STR) { str(); return; }
        int w = scalar_width(t);
        if (w <= 0) { bad = true; return; }
        if (need((size_t)w)) off += (size_t)w;
    }
    void skip(uint32_t t) {
        if (t != T_ARR) { skip_scalar(t); return; }
        uint32_t et = get<uint32_t>();
        uint64_t cnt = get<uint64_t>();
        for (uint64_t i = 0; i < cnt && !bad; i++) skip_scalar(et);
    }
};

// key == arch + "." + suffix
bool is_key(const std::string &key, const std::string &arch, const char *suffix) {
    size_t a = arch.size(), s = strlen(suffix);
    return key.size() == a + 1 + s && key.compare(0, a, arch) == 0 && key[a] == '.' &&
           key.compare(a + 1, s, suffix) == 0;
}

struct Mapped {
    void  *base = nullptr;
    size_t size = 0;
};

int map_file(const char *path, Mapped &m) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return CMOL_ERR_IO;
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) { close(fd); return CMOL_ERR_IO; }
    void *b = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (b == MAP_FAILED) return CMOL_ERR_IO;
    m.base = b;
    m.size = (size_t)st.st_size;
    return CMOL_OK;
}

// Parse header + KV section.  `full` also reads the tokenizer arrays.
int parse_kv(Reader &r, HParams &hp, HVocab *voc, uint64_t &n_tensors, uint32_t &align) {
    uint32_t magic = r.get<uint32_t>();
    uint32_t version = r.get<uint32_t>();
    if (r.bad || magic != 0x46554747u) return CMOL_ERR_INVALID;
    if (version < 2 || version > 3) return CMOL_ERR_UNSUPPORTED;
    n_tensors = r.get<uint64_t>();
    uint64_t n_kv = r.get<uint64_t>();
    if (r.bad || n_tensors > 65536 || n_kv > 65536) return CMOL_ERR_INVALID;
    hp = HParams();
    align = 32;
    for (uint64_t i = 0; i < n_kv && !r.bad; i++) {
        std::string key = r.str();
        uint32_t t = r.get<uint32_t>();
        if (r.bad) break;
        if (key == "general.architecture" && t == T_STR) { hp.arch = r.str(); continue; }
        if (t == T_U32) {
            uint32_t v = r.get<uint32_t>();
            if (is_key(key, hp.arch, "context_length")) hp.model_max_ctx = (int)v;
            else if (is_key(key, hp.arch, "embedding_length")) hp.d_model = (int)v;
            else if (is_key(key, hp.arch, "block_count")) hp.n_layers = (int)v;
            else if (is_key(key, hp.arch, "feed_forward_length")) hp.d_ffn = (int)v;
            else if (is_key(key, hp.arch, "attention.head_count")) hp.n_heads = (int)v;
            else if (is_key(key, hp.arch, "attention.head_count_kv")) hp.n_kv_heads = (int)v;
            else if (is_key(key, hp.arch, "vocab_size")) hp.vocab_size = (int)v;
            else if (is_key(key, hp.arch, "attention.no_rope_layer_interval")) hp.no_rope_layer_interval = (int)v;
            else if (key == "general.alignment") align = v ? v : 32;
            else if (voc && key == "tokenizer.ggml.bos_token_id") voc->bos = (int32_t)v;
            else if (voc && key == "tokenizer.ggml.eos_token_id") voc->eos = (int32_t)v;
            else if (voc && key == "tokenizer.ggml.unknown_token_id") voc->unk = (int32_t)v;
            continue;
        }
        if (t == T_F32) {
            float v = r.get<float>();
            if (is_key(key, hp.arch, "rope.freq_base")) hp.rope_freq_base = v;
            else if (is_key(key, hp.arch, "attention.layer_norm_rms_epsilon")) hp.rms_norm_eps = v;
            continue;
        }
        if (t == T_BOOL) {
            uint8_t v = r.get<uint8_t>();
            if (voc && key == "tokenizer.ggml.add_bos_token") voc->add_bos = v ? 1 : 0;
            continue;
        }
        if (t == T_STR && voc && key == "tokenizer.ggml.model") {
            voc->gpt2 = r.str() != "llama";
            continue;
        }
        if (t == T_STR && is_key(key, hp.arch, "rope.scaling.type")) {
            r.str();
            hp.yarn_factor_x100 = -1;   // recorded, not applied (as the reference)
            continue;
        }
        if (t == T_ARR && voc) {
            size_t save = r.off;
            uint32_t et = r.get<uint32_t>();
            uint64_t cnt = r.get<uint64_t>();
            if (r.bad) break;
            if (cnt > r.n) { r.bad = true; break; }
            if (key == "tokenizer.ggml.tokens" && et == T_STR) {
                voc->tokens.resize((size_t)cnt);
                for (uint64_t j = 0; j < cnt && !r.bad; j++) voc->tokens[j] = r.str();
                continue;
            }
            if (key == "tokenizer.ggml.merges" && et == T_STR) {
                voc->merges.resize((size_t)cnt);
                for (uint64_t j = 0; j < cnt && !r.bad; j++) voc->merges[j] = r.str();
                continue;
            }
            if (key == "tokenizer.ggml.scores" && et == T_F32) {
                voc->scores.resize((size_t)cnt);
                for (uint64_t j = 0; j < cnt && !r.bad; j++) voc->scores[j] = r.get<float>();
                continue;
            }
            if (key == "tokenizer.ggml.token_type" && et == T_I32) {
                voc->types.resize((size_t)cnt);
                for (uint64_t j = 0; j < cnt && !r.bad; j++) voc->types[j] = (uint8_t)r.get<int32_t>();
                continue;
            }
            r.off = save;
        }
        r.skip(t);
    }
    if (r.bad) return CMOL_ERR_INVALID;
    if (hp.n_kv_heads == 0) hp.n_kv_heads = hp.n_heads;
    if (hp.n_heads > 0) hp.d_head = hp.d_model / hp.n_heads;
    return CMOL_OK;
}

}  // namespace

size_t dtype_row_bytes(int dtype, int64_t k) {
    switch (dtype) {
    case 0: return (size_t)k * 4;
    case 1: return (size_t)k * 2;
    case 2: return (size_t)(k / 32) * 18;
    case 6: return (size_t)(k / 32) * 22;
    case 8: return (size_t)(k / 32) * 34;
    case 12: return (size_t)(k / 256) * 144;
    case 14: return (size_t)(k / 256) * 210;
    default: return 0;
    }
}

const HTensor *HostModel::find(const std::string &name) const {
    for (const HTensor &t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}

const HTensor *HostModel::blk(int layer, const char *suffix) const {
    return find("blk." + std::to_string(layer) + "." + suffix);
}

HostModel::~HostModel() {
    if (map) munmap(map, map_size);
}

int gguf_peek(const char *path, HParams &hp, size_t &n_tensors) {
    Mapped mm;
    int rc = map_file(path, mm);
    if (rc) return rc;
    Reader r{(const uint8_t *)mm.base, mm.size};
    uint64_t nt = 0;
    uint32_t align = 32;
    rc = parse_kv(r, hp, nullptr, nt, align);
    munmap(mm.base, mm.size);
    if (rc) return rc;
    n_tensors = (size_t)nt;
    return CMOL_OK;
}

int gguf_load(const char *path, HostModel &m) {
    Mapped mm;
    int rc = map_file(path, mm);
    if (rc) return rc;
    m.map = mm.base;
    m.map_size = mm.size;
    Reader r{(const uint8_t *)mm.base, mm.size};
    uint64_t nt = 0;
    uint32_t align = 32;
    rc = parse_kv(r, m.hp, &m.vocab, nt, align);
    if (rc) return rc;
    if (m.hp.vocab_size == 0) m.hp.vocab_size = (int)m.vocab.tokens.size();
    m.tensors.resize((size_t)nt);
    std::vector<uint64_t> offs((size_t)nt);
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        HTensor &t = m.tensors[i];
        t.name = r.str();
        uint32_t nd = r.get<uint32_t>();
        if (r.bad || nd < 1 || nd > 4) return CMOL_ERR_INVALID;
        t.n_dims = (int)nd;
        int64_t ne = 1;
        for (uint32_t d = 0; d < nd; d++) {
            t.dims[d] = (int64_t)r.get<uint64_t>();
            ne *= t.dims[d];
        }
        t.dtype = (int)r.get<uint32_t>();
        offs[i] = r.get<uint64_t>();
        size_t rb = dtype_row_bytes(t.dtype, t.dims[0]);
        t.nbytes = ne > 0 && t.dims[0] > 0 ? rb * (size_t)(ne / t.dims[0]) : 0;
    }
    if (r.bad) return CMOL_ERR_INVALID;
    size_t data0 = (r.off + align - 1) / align * align;
    for (uint64_t i = 0; i < nt; i++) {
        HTensor &t = m.tensors[i];
        size_t off = data0 + (size_t)offs[i];
        if (off > mm.size || t.nbytes > mm.size - off) return CMOL_ERR_INVALID;
        t.data = (const uint8_t *)mm.base + off;
    }
    m.hp.tie_embeddings = m.find("output.weight") == nullptr;
    return CMOL_OK;
}

}  // namespace cmolrt
