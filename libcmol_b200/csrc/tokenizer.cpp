// tokenizer.cpp — see tokenizer.h.
#include "tokenizer.h"

#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <queue>

#include "cmol.h"

namespace cmolrt {

namespace {

const int kWorkMax = 4096;              // initial symbols per encode (src/tokenizer.c:354)
const char kSpiece[] = "\xe2\x96\x81";  // U+2581
enum { TT_NORMAL = 1, TT_UNKNOWN = 2, TT_CONTROL = 3, TT_BYTE = 6 };

int utf8_len(unsigned char c) {
    if ((c & 0x80) == 0x00) return 1;
    if ((c & 0xE0) == 0xC0) return 2;
    if ((c & 0xF0) == 0xE0) return 3;
    if ((c & 0xF8) == 0xF0) return 4;
    return 1;
}

// GPT-2 byte <-> codepoint map (printable bytes map to themselves, the other
// 68 bytes to U+0100.. in byte order).
unsigned gpt2_cp(unsigned char b) {
    if (b <= 0x20) return 0x100u + b;
    if (b <= 0x7E) return b;
    if (b == 0x7F) return 0x121u;
    if (b <= 0xA0) return 0x122u + (b - 0x80u);
    if (b == 0xAD) return 0x143u;
    return b;
}

unsigned char gpt2_byte(unsigned cp) {
    if (cp >= 0x100 && cp <= 0x120) return (unsigned char)(cp - 0x100);
    if (cp == 0x121) return 0x7F;
    if (cp >= 0x122 && cp <= 0x142) return (unsigned char)(0x80 + (cp - 0x122));
    if (cp == 0x143) return 0xAD;
    return (unsigned char)(cp & 0xFF);
}

void put_utf8(unsigned cp, std::string &o) {
    if (cp < 0x80) { o += (char)cp; }
    else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) {
        o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F));
    } else {
        o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F));
        o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F));
    }
}

// Next codepoint of a NUL-terminated string; 0 at the end.
unsigned next_cp(const char *&p) {
    const unsigned char *u = (const unsigned char *)p;
    if (!*u) return 0;
    unsigned cp;
    int n;
    if (u[0] < 0x80) { cp = u[0]; n = 1; }
    else if (u[0] < 0xC0) { p++; return 0xFFFD; }
    else if (u[0] < 0xE0) { cp = u[0] & 0x1F; n = 2; }
    else if (u[0] < 0xF0) { cp = u[0] & 0x0F; n = 3; }
    else { cp = u[0] & 0x07; n = 4; }
    int i = 1;
    for (; i < n; i++) {
        if ((u[i] & 0xC0) != 0x80) break;
        cp = (cp << 6) | (u[i] & 0x3F);
    }
    p += i;   // stop at a truncated sequence instead of running past the end
    return cp;
}

}  // namespace

int32_t Tokenizer::find(const std::string &s) const {
    auto it = index_.find(s);
    return it == index_.end() ? -1 : it->second;
}

int32_t Tokenizer::merge_rank(int32_t l, int32_t r) const {
    if (l < 0 || r < 0) return -1;
    auto it = rank_.find(((uint64_t)(uint32_t)l << 32) | (uint32_t)r);
    return it == rank_.end() ? -1 : it->second;
}

int Tokenizer::build(const HVocab &v, int vocab_size) {
    const int V = (int)v.tokens.size();
    if (V == 0) return CMOL_ERR_INVALID;
    (void)vocab_size;
    vocab_ = v.tokens;
    types_ = v.types;
    bos_ = v.bos; eos_ = v.eos; unk_ = v.unk; add_bos_ = v.add_bos; gpt2_ = v.gpt2;
    index_.reserve((size_t)V * 2);
    for (int i = 0; i < V; i++) index_.emplace(vocab_[i], i);   // first occurrence wins
    // merges "L R" split at the first space (src/gguf.c:260-289)
    const int M = (int)v.merges.size();
    merge_result_.assign((size_t)M, unk_);
    rank_.reserve((size_t)M * 2);
    for (int i = 0; i < M; i++) {
        const std::string &s = v.merges[i];
        size_t sp = s.find(' ');
        if (sp == std::string::npos || sp >= 512) continue;
        int32_t l = find(s.substr(0, sp)), r = find(s.substr(sp + 1));
        if (l < 0 || r < 0) continue;
        rank_.emplace(((uint64_t)(uint32_t)l << 32) | (uint32_t)r, i);
        const std::string cat = vocab_[l] + vocab_[r];
        if (cat.size() < 256) {
            int32_t id = find(cat);
            merge_result_[i] = id >= 0 ? id : unk_;
        }
    }
    // control tokens, longest first then lowest id
    for (int i = 0; i < V && i < (int)types_.size(); i++)
        if (types_[i] == TT_CONTROL && !vocab_[i].empty()) controls_.push_back(i);
    std::stable_sort(controls_.begin(), controls_.end(),
                     [&](int32_t a, int32_t b) { return vocab_[a].size() > vocab_[b].size(); });
    // output forms (src/tokenizer.c:253-340)
    decoded_.resize((size_t)V);
    for (int i = 0; i < V; i++) {
        const std::string &s = vocab_[i];
        if (gpt2_) {
            bool ctrl = i < (int)types_.size() && types_[i] == TT_CONTROL;
            std::string d;
            if (!ctrl) {
                const char *p = s.c_str();
                while (*p && d.size() < 255) {
                    unsigned cp = next_cp(p);
                    if (!cp) break;
                    d += (char)gpt2_byte(cp);
                }
            }
            decoded_[i] = (!ctrl && !d.empty()) ? d : s;
            continue;
        }
        bool is_byte = i < (int)types_.size() && types_[i] == TT_BYTE;
        if (!is_byte && s.size() == 6 && s[0] == '<' && s[1] == '0' && s[2] == 'x' && s[5] == '>') is_byte = true;
        if (is_byte) {
            unsigned bv = 0;
            if (sscanf(s.c_str(), "<0x%02x>", &bv) == 1) {
                decoded_[i] = std::string(1, (char)(unsigned char)bv);
                continue;
            }
        }
        if (s.size() >= 3 && s.compare(0, 3, kSpiece) == 0) {
            decoded_[i] = " " + s.substr(3);
            continue;
        }
        decoded_[i] = s;
    }
    return CMOL_OK;
}

const char *Tokenizer::decode(int32_t id) const {
    if (id < 0 || id >= (int32_t)decoded_.size()) return nullptr;
    return decoded_[id].c_str();   // a byte token 0x00 decodes to "" (length 0)
}

int Tokenizer::encode(const char *text, int32_t *out, int cap, int add_bos) const {
    if (!text || !out || cap <= 0) return CMOL_ERR_ARGS;
    int n = 0;
    if (add_bos && bos_ >= 0) out[n++] = bos_;
    std::vector<int32_t> work;
    work.reserve(256);
    bool overflow = false;
    auto push = [&](int32_t id) {
        if ((int)work.size() < kWorkMax) work.push_back(id);
        else overflow = true;
    };
    // vocabulary lookup of one character, byte tokens on a miss (the byte
    // token names are formatted lower-case, as the reference does)
    auto emit_char = [&](const char *p, int len) {
        int32_t id = find(std::string(p, (size_t)len));
        if (id >= 0) { push(id); return; }
        for (int b = 0; b < len && !overflow; b++) {
            char bt[8];
            snprintf(bt, sizeof bt, "<0x%02x>", (unsigned char)p[b]);
            int32_t bid = find(bt);
            if (bid < 0) bid = unk_;
            if (bid >= 0) push(bid);
        }
    };
    auto match_control = [&](const char *p, size_t &len) -> int32_t {
        for (int32_t id : controls_) {
            const std::string &c = vocab_[id];
            if (strncmp(p, c.c_str(), c.size()) == 0) { len = c.size(); return id; }
        }
        return -1;
    };
    const char *p = text;
    if (gpt2_) {
        while (*p && !overflow) {
            size_t cl = 0;
            int32_t cid = types_.empty() ? -1 : match_control(p, cl);
            if (cid >= 0) { push(cid); p += cl; continue; }
            std::string u;
            put_utf8(gpt2_cp((unsigned char)*p++), u);
            int32_t id = find(u);
            if (id < 0) id = unk_;
            if (id >= 0) push(id);
        }
    } else {
        bool prefix_done = false;
        while (*p && !overflow) {
            size_t cl = 0;
            int32_t cid = types_.empty() ? -1 : match_control(p, cl);
            if (cid >= 0) { push(cid); p += cl; prefix_done = false; continue; }
            if (!prefix_done) { emit_char(kSpiece, 3); prefix_done = true; }
            if (*p == ' ') { emit_char(kSpiece, 3); p++; continue; }
            int len = utf8_len((unsigned char)*p);
            int avail = (int)strnlen(p, (size_t)len);
            if (len > avail) len = avail;
            emit_char(p, len);
            p += len;
        }
    }
    // BPE merges: lowest rank first, leftmost among equal ranks
    const int w = (int)work.size();
    if (!rank_.empty() && w > 1) {
        std::vector<int32_t> tok(work);
        std::vector<int> nxt(w), prv(w);
        std::vector<char> alive(w, 1);
        for (int i = 0; i < w; i++) { nxt[i] = i + 1 < w ? i + 1 : -1; prv[i] = i - 1; }
        typedef std::pair<int32_t, int> Key;   // (rank, left symbol index)
        std::priority_queue<Key, std::vector<Key>, std::greater<Key>> pq;
        auto consider = [&](int i) {
            if (i < 0 || !alive[i] || nxt[i] < 0) return;
            int32_t r = merge_rank(tok[i], tok[nxt[i]]);
            if (r >= 0) pq.push(Key(r, i));
        };
        for (int i = 0; i + 1 < w; i++) consider(i);
        while (!pq.empty()) {
            Key k = pq.top();
            pq.pop();
            int i = k.second;
            if (!alive[i] || nxt[i] < 0) continue;
            if (merge_rank(tok[i], tok[nxt[i]]) != k.first) continue;   // stale entry
            int j = nxt[i];
            tok[i] = merge_result_[(size_t)k.first];
            alive[j] = 0;
            nxt[i] = nxt[j];
            if (nxt[j] >= 0) prv[nxt[j]] = i;
            consider(prv[i]);
            consider(i);
        }
        work.clear();
        for (int i = 0; i >= 0 && i < w; i = nxt[i]) work.push_back(tok[i]);
    }
    bool trunc = overflow;
    for (int32_t id : work) {
        if (n >= cap) { trunc = true; break; }
        out[n++] = id;
    }
    return trunc ? CMOL_ERR_TRUNC : n;
}

}  // namespace cmolrt
