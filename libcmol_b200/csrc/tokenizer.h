// tokenizer.h — SentencePiece-style BPE with byte fallback (host C++).
//
// Same observable behaviour as the reference tokenizer
// (src/tokenizer.c:189-571 of nvlass/libcmol): control tokens matched
// verbatim (longest first) and emitted directly; a U+2581 prefix injected
// at the start of every text segment; spaces become U+2581; each UTF-8
// character looked up in the vocabulary, with <0xNN> byte tokens on a miss;
// merges applied lowest rank first, leftmost among equal ranks; at most
// 4096 initial symbols (CMOL_ERR_TRUNC beyond).  GPT-2 vocabularies use the
// byte-to-unicode mapping for both directions.  The merge loop here keeps a
// heap of candidate pairs, so it runs in O(w log w) instead of O(w^2) and
// gives the same merges.
#pragma once
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "host_model.h"

namespace cmolrt {

class Tokenizer {
  public:
    int  build(const HVocab &v, int vocab_size);   // cmol_err_t
    int  encode(const char *text, int32_t *out, int cap, int add_bos) const;
    const char *decode(int32_t id) const;
    int32_t bos() const { return bos_; }
    int32_t eos() const { return eos_; }
    int     add_bos() const { return add_bos_; }

  private:
    int32_t find(const std::string &s) const;
    int32_t merge_rank(int32_t l, int32_t r) const;

    std::vector<std::string>              vocab_;
    std::vector<std::string>              decoded_;
    std::vector<uint8_t>                  types_;
    std::unordered_map<std::string, int32_t> index_;
    std::unordered_map<uint64_t, int32_t>    rank_;     // (l << 32 | r) -> merge rank
    std::vector<int32_t>                  merge_result_;
    std::vector<int32_t>                  controls_;    // control-token ids
    int32_t bos_ = -1, eos_ = -1, unk_ = -1;
    int     add_bos_ = 1;
    int     gpt2_ = 0;
};

}  // namespace cmolrt
