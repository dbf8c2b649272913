// host_model.h — the GGUF file as the host runtime sees it (no CUDA types).
//
// The parser follows the behaviour of the reference loader
// (src/gguf.c:448-518 and cmol_gguf_peek, src/gguf.c:535-626 of
// nvlass/libcmol): GGUF v2/v3, architecture-prefixed keys matched against
// general.architecture, the same defaults (rope base 1e4, eps 1e-5, token
// ids -1, add_bos 1), n_kv_heads defaulting to n_heads, d_head = d_model /
// n_heads, tied embeddings when output.weight is absent.  Differences: the
// tensor data section honours general.alignment when present (default 32),
// and Q4_0 tensors are sized (18 bytes per 32 values).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace cmolrt {

struct HTensor {
    std::string    name;
    int            dtype = 0;
    int            n_dims = 0;
    int64_t        dims[4] = {1, 1, 1, 1};   // dims[0] innermost
    const uint8_t *data = nullptr;          // into the mmap
    size_t         nbytes = 0;
};

struct HParams {
    int         n_layers = 0, n_heads = 0, n_kv_heads = 0, d_model = 0, d_head = 0;
    int         d_ffn = 0, vocab_size = 0, model_max_ctx = 0;
    float       rope_freq_base = 10000.0f, rms_norm_eps = 1e-5f;
    int         no_rope_layer_interval = 0;
    int         yarn_factor_x100 = 0;
    int         tie_embeddings = 0;
    std::string arch = "llama";
};

struct HVocab {
    std::vector<std::string> tokens;
    std::vector<float>       scores;
    std::vector<uint8_t>     types;
    std::vector<std::string> merges;
    int32_t bos = -1, eos = -1, unk = -1;
    int     add_bos = 1;
    int     gpt2 = 0;          // tokenizer.ggml.model != "llama"
};

struct HostModel {
    HParams              hp;
    HVocab               vocab;
    std::vector<HTensor> tensors;
    void                *map = nullptr;
    size_t               map_size = 0;

    const HTensor *find(const std::string &name) const;
    const HTensor *blk(int layer, const char *suffix) const;
    ~HostModel();
};

size_t dtype_row_bytes(int dtype, int64_t k);   // 0 for unknown types

// Returns a cmol_err_t value (0 = OK).
int gguf_load(const char *path, HostModel &m);
int gguf_peek(const char *path, HParams &hp, size_t &n_tensors);

}  // namespace cmolrt
