// sd_tokenizer.cu -- host-side SentencePiece-style BPE tokenizer over a GGUF vocabulary (no device code).
//
// Replaces mistral/tokenizer.h:
//   tokenizer_init          :121-153  vocabulary, scores and token types of the GGUF (tokenizer.ggml.*)
//   tokenizer_encode        :200-346  " " + text, spaces as U+2581, one piece per UTF-8 character (byte fallback
//                                     <0xNN> for characters outside the vocabulary), then merges of adjacent
//                                     pieces in order of the merged piece's score
//   tokenizer_decode_token  :348-373
//   tokenizer_decode        :375-412
//   tokenizer_apply_chat    :416-429  "[INST] {msg} [/INST]"
// Token ids must equal the reference's for every input, so two behaviours are kept alike on purpose:
//   - merge candidates wait in a binary max-heap keyed by score whose ties resolve as the reference's heap
//     resolves them (push: sift up while the parent's score is strictly lower; pop: the last element moves to
//     the root and sinks toward the larger child, the left one on equal scores, while a child is strictly
//     larger).  Equal-score merges at different positions are applied in that order.
//   - a piece that stayed a byte-fallback token is emitted as the byte tokens of every byte of its original
//     character.
// Lookups skip CONTROL and UNKNOWN tokens and return the lowest id among equal strings.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "sd_host.h"
#include "specdec_b200.h"

namespace {

enum : int { kTokNormal = 1, kTokUnknown = 2, kTokControl = 3, kTokUnused = 4, kTokByte = 6 };

// GGUF value types (the subset the vocabulary uses; gguf_loader.h:24-37)
enum : uint32_t { GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STR, GT_ARR, GT_U64, GT_I64, GT_F64 };

struct Reader {
    const uint8_t* b;
    size_t pos, len;
    bool ok = true;
    bool need(size_t n) {
        if (pos + n > len) ok = false;
        return ok;
    }
    uint64_t u(int n) {
        if (!need((size_t)n)) return 0;
        uint64_t v = 0;
        memcpy(&v, b + pos, (size_t)n);
        pos += (size_t)n;
        return v;
    }
    std::string str() {
        const uint64_t n = u(8);
        if (!need((size_t)n)) return std::string();
        std::string s(reinterpret_cast<const char*>(b) + pos, (size_t)n);
        pos += (size_t)n;
        return s;
    }
};

int scalar_size(uint32_t t) {
    switch (t) {
        case GT_U8: case GT_I8: case GT_BOOL: return 1;
        case GT_U16: case GT_I16: return 2;
        case GT_U32: case GT_I32: case GT_F32: return 4;
        case GT_U64: case GT_I64: case GT_F64: return 8;
        default: return -1;
    }
}

void skip_value(Reader& r, uint32_t t, int depth = 0) {
    if (t == GT_STR) {
        const uint64_t n = r.u(8);
        if (r.need((size_t)n)) r.pos += (size_t)n;
    } else if (t == GT_ARR) {
        const uint32_t at = (uint32_t)r.u(4);
        const uint64_t n = r.u(8);
        if (depth > 2) { r.ok = false; return; }
        const int es = scalar_size(at);
        if (es > 0) {
            if (r.need((size_t)(n * (uint64_t)es))) r.pos += (size_t)(n * (uint64_t)es);
        } else {
            for (uint64_t i = 0; i < n && r.ok; ++i) skip_value(r, at, depth + 1);
        }
    } else {
        const int es = scalar_size(t);
        if (es < 0) r.ok = false;
        else if (r.need((size_t)es)) r.pos += (size_t)es;
    }
}

int64_t scalar_int(Reader& r, uint32_t t) {
    switch (t) {
        case GT_U8: return (int64_t)r.u(1);
        case GT_I8: return (int8_t)r.u(1);
        case GT_U16: return (int64_t)r.u(2);
        case GT_I16: return (int16_t)r.u(2);
        case GT_U32: return (int64_t)r.u(4);
        case GT_I32: return (int32_t)r.u(4);
        case GT_U64: return (int64_t)r.u(8);
        case GT_I64: return (int64_t)r.u(8);
        default: skip_value(r, t); return 0;
    }
}

int utf8_len(uint8_t c) { return c < 0x80 ? 1 : c < 0xE0 ? 2 : c < 0xF0 ? 3 : 4; }

// A merge candidate: the pieces at node `pos` and its right neighbour, as they were when it was pushed.
struct Cand {
    float score;
    int pos, left, right;
};

// Binary max-heap on score with the tie behaviour described at the top of this file.
struct CandHeap {
    std::vector<Cand> v;
    void push(const Cand& c) {
        v.push_back(c);
        size_t i = v.size() - 1;
        while (i > 0) {
            const size_t p = (i - 1) / 2;
            if (!(v[p].score < v[i].score)) break;
            std::swap(v[p], v[i]);
            i = p;
        }
    }
    Cand pop() {
        const Cand top = v[0];
        v[0] = v.back();
        v.pop_back();
        size_t i = 0;
        const size_t n = v.size();
        for (;;) {
            size_t b = i;
            const size_t l = 2 * i + 1, r = 2 * i + 2;
            if (l < n && v[l].score > v[b].score) b = l;
            if (r < n && v[r].score > v[b].score) b = r;
            if (b == i) break;
            std::swap(v[i], v[b]);
            i = b;
        }
        return top;
    }
};

}  // namespace

struct sd_tokenizer {
    std::vector<std::string> piece;
    std::vector<float> score;
    std::vector<int> type;
    std::unordered_map<std::string, int> lookup;  // non-CONTROL / non-UNKNOWN pieces -> lowest id
    int bos = 1, eos = 2;

    int find(const char* s, size_t n) const {
        auto it = lookup.find(std::string(s, n));
        return it == lookup.end() ? -1 : it->second;
    }
    int byte_token(uint8_t byte) const {
        char buf[8];
        snprintf(buf, sizeof buf, "<0x%02X>", byte);
        const int id = find(buf, strlen(buf));
        return id >= 0 ? id : 0;
    }
};

namespace {
using sd::fail;

int parse_vocab(const void* base, size_t len, sd_tokenizer& t) {
    Reader r{static_cast<const uint8_t*>(base), 0, len};
    if (r.u(4) != 0x46554747u) return fail(SD_ERR_FORMAT, "tokenizer: not a GGUF image");
    const uint32_t ver = (uint32_t)r.u(4);
    if (ver < 2) return fail(SD_ERR_FORMAT, "tokenizer: GGUF version %u unsupported", ver);
    r.u(8);  // tensor count
    const uint64_t n_kv = r.u(8);
    if (!r.ok || n_kv > 100000) return fail(SD_ERR_FORMAT, "tokenizer: GGUF header truncated");
    bool have_tokens = false;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string k = r.str();
        const uint32_t vt = (uint32_t)r.u(4);
        if (k == "tokenizer.ggml.tokens" && vt == GT_ARR) {
            const uint32_t at = (uint32_t)r.u(4);
            const uint64_t n = r.u(8);
            if (at != GT_STR || n > (1u << 24)) return fail(SD_ERR_FORMAT, "tokenizer: bad token array");
            t.piece.resize((size_t)n);
            for (uint64_t j = 0; j < n && r.ok; ++j) t.piece[j] = r.str();
            have_tokens = true;
        } else if (k == "tokenizer.ggml.scores" && vt == GT_ARR) {
            const uint32_t at = (uint32_t)r.u(4);
            const uint64_t n = r.u(8);
            if (at != GT_F32 || n > (1u << 24)) return fail(SD_ERR_FORMAT, "tokenizer: bad score array");
            t.score.resize((size_t)n);
            if (r.need((size_t)n * 4)) {
                memcpy(t.score.data(), r.b + r.pos, (size_t)n * 4);
                r.pos += (size_t)n * 4;
            }
        } else if (k == "tokenizer.ggml.token_type" && vt == GT_ARR) {
            const uint32_t at = (uint32_t)r.u(4);
            const uint64_t n = r.u(8);
            if (n > (1u << 24)) return fail(SD_ERR_FORMAT, "tokenizer: bad token type array");
            t.type.resize((size_t)n);
            for (uint64_t j = 0; j < n && r.ok; ++j) t.type[j] = (int)scalar_int(r, at);
        } else if (k == "tokenizer.ggml.bos_token_id") {
            t.bos = (int)scalar_int(r, vt);
        } else if (k == "tokenizer.ggml.eos_token_id") {
            t.eos = (int)scalar_int(r, vt);
        } else {
            skip_value(r, vt);
        }
    }
    if (!r.ok) return fail(SD_ERR_FORMAT, "tokenizer: GGUF metadata truncated");
    if (!have_tokens || t.piece.empty()) return fail(SD_ERR_FORMAT, "tokenizer: the GGUF has no tokenizer.ggml.tokens");
    const size_t n = t.piece.size();
    if (t.score.size() != n) t.score.assign(n, 0.0f);     // absent scores read as 0 (tokenizer.h:135)
    if (t.type.size() != n) t.type.assign(n, kTokNormal);  // absent types read as NORMAL (tokenizer.h:136)
    t.lookup.reserve(n * 2);
    for (size_t i = 0; i < n; ++i)
        if (t.type[i] != kTokControl && t.type[i] != kTokUnknown) t.lookup.emplace(t.piece[i], (int)i);
    return SD_OK;
}

struct Node {
    int id, prev, next;
};

void try_merge(const sd_tokenizer& t, const std::vector<Node>& nodes, int left, int right, CandHeap& heap) {
    if (left < 0 || right < 0) return;
    const std::string& a = t.piece[nodes[left].id];
    const std::string& b = t.piece[nodes[right].id];
    if (a.size() + b.size() > 256) return;
    const int m = t.find((a + b).data(), a.size() + b.size());
    if (m >= 0) heap.push(Cand{t.score[m], left, nodes[left].id, nodes[right].id});
}

}  // namespace

extern "C" {

int sd_tokenizer_create(const void* gguf_base, size_t gguf_len, sd_tokenizer** out) {
    sd::clear_error();
    if (!gguf_base || !out) return fail(SD_ERR_INVALID, "sd_tokenizer_create: null argument");
    *out = nullptr;
    sd_tokenizer* t = new (std::nothrow) sd_tokenizer();
    if (!t) return fail(SD_ERR_OOM, "sd_tokenizer_create: out of memory");
    const int rc = parse_vocab(gguf_base, gguf_len, *t);
    if (rc != SD_OK) {
        delete t;
        return rc;
    }
    *out = t;
    return SD_OK;
}

void sd_tokenizer_free(sd_tokenizer* t) { delete t; }

int sd_tokenizer_info(const sd_tokenizer* t, int* vocab_size, int* bos_id, int* eos_id) {
    if (!t) return fail(SD_ERR_INVALID, "sd_tokenizer_info: null tokenizer");
    if (vocab_size) *vocab_size = (int)t->piece.size();
    if (bos_id) *bos_id = t->bos;
    if (eos_id) *eos_id = t->eos;
    return SD_OK;
}

int sd_tokenizer_entry(const sd_tokenizer* t, int id, const char** piece, float* score, int* type) {
    if (!t || id < 0 || id >= (int)t->piece.size()) return fail(SD_ERR_INVALID, "sd_tokenizer_entry: bad id");
    if (piece) *piece = t->piece[id].c_str();
    if (score) *score = t->score[id];
    if (type) *type = t->type[id];
    return SD_OK;
}

int sd_tokenizer_encode(const sd_tokenizer* t, const char* text, int32_t* out, int max_tokens, int add_bos) {
    sd::clear_error();
    if (!t || !out || max_tokens < 0) return fail(SD_ERR_INVALID, "sd_tokenizer_encode: bad arguments");
    int n = 0;
    if (add_bos && n < max_tokens) out[n++] = t->bos;
    if (!text || !*text) return n;
    const std::string work = std::string(" ") + text;
    // one piece per UTF-8 character (a lead byte's length, cut at the end of the text); ' ' becomes U+2581
    std::vector<std::string> chars;
    for (size_t i = 0; i < work.size();) {
        const uint8_t c = (uint8_t)work[i];
        if (c == ' ') {
            chars.emplace_back("\xE2\x96\x81");
            ++i;
        } else {
            size_t l = (size_t)utf8_len(c);
            if (i + l > work.size()) l = work.size() - i;
            chars.emplace_back(work.substr(i, l));
            i += l;
        }
    }
    const int nc = (int)chars.size();
    std::vector<Node> nodes((size_t)nc);
    for (int c = 0; c < nc; ++c) {
        const int id = t->find(chars[c].data(), chars[c].size());
        nodes[c].id = id >= 0 ? id : t->byte_token((uint8_t)chars[c][0]);
        nodes[c].prev = c - 1;
        nodes[c].next = c + 1 < nc ? c + 1 : -1;
    }
    CandHeap heap;
    for (int c = 0; c + 1 < nc; ++c) try_merge(*t, nodes, c, nodes[c].next, heap);
    while (!heap.v.empty()) {
        const Cand m = heap.pop();
        if (nodes[m.pos].id != m.left) continue;
        const int right = nodes[m.pos].next;
        if (right < 0 || nodes[right].id != m.right) continue;
        const std::string& a = t->piece[m.left];
        const std::string& b = t->piece[m.right];
        const int merged = t->find((a + b).data(), a.size() + b.size());
        if (merged < 0) continue;
        nodes[m.pos].id = merged;
        nodes[m.pos].next = nodes[right].next;
        if (nodes[right].next >= 0) nodes[nodes[right].next].prev = m.pos;
        if (nodes[m.pos].prev >= 0) try_merge(*t, nodes, nodes[m.pos].prev, m.pos, heap);
        if (nodes[m.pos].next >= 0) try_merge(*t, nodes, m.pos, nodes[m.pos].next, heap);
    }
    for (int cur = 0; cur >= 0 && n < max_tokens; cur = nodes[cur].next) {
        const int id = nodes[cur].id;
        if (t->type[id] == kTokByte) {
            // a byte-fallback piece: every byte of the character it stood for (node index = character index)
            for (size_t b = 0; b < chars[cur].size() && n < max_tokens; ++b)
                out[n++] = t->byte_token((uint8_t)chars[cur][b]);
        } else {
            out[n++] = id;
        }
    }
    return n;
}

const char* sd_tokenizer_piece(const sd_tokenizer* t, int id) {
    static thread_local char byte_buf[2];
    if (!t || id < 0 || id >= (int)t->piece.size()) return "";
    if (id == t->bos || id == t->eos) return "";
    const std::string& s = t->piece[id];
    if (t->type[id] == kTokByte && s.size() >= 3 && s[0] == '<' && s[1] == '0' && s[2] == 'x') {
        unsigned v = 0;
        for (size_t i = 3; i < s.size() && s[i] != '>'; ++i) {
            const char c = s[i];
            v <<= 4;
            if (c >= '0' && c <= '9') v += (unsigned)(c - '0');
            else if (c >= 'A' && c <= 'F') v += (unsigned)(c - 'A' + 10);
            else if (c >= 'a' && c <= 'f') v += (unsigned)(c - 'a' + 10);
        }
        byte_buf[0] = (char)v;
        byte_buf[1] = '\0';
        return byte_buf;
    }
    return s.c_str();
}

char* sd_tokenizer_decode(const sd_tokenizer* t, const int32_t* tokens, int n) {
    std::string out;
    for (int i = 0; t && tokens && i < n; ++i) {
        const char* p = sd_tokenizer_piece(t, tokens[i]);
        const size_t l = strlen(p);
        for (size_t j = 0; j < l;) {
            if (j + 2 < l && (uint8_t)p[j] == 0xE2 && (uint8_t)p[j + 1] == 0x96 && (uint8_t)p[j + 2] == 0x81) {
                out.push_back(' ');
                j += 3;
            } else {
                out.push_back(p[j++]);
            }
        }
    }
    if (!out.empty() && out[0] == ' ') out.erase(0, 1);  // the space the encoder prepended
    char* r = static_cast<char*>(malloc(out.size() + 1));
    if (r) memcpy(r, out.c_str(), out.size() + 1);
    return r;
}

char* sd_tokenizer_apply_chat(const char* user_msg) {
    const std::string s = std::string("[INST] ") + (user_msg ? user_msg : "") + " [/INST]";
    char* r = static_cast<char*>(malloc(s.size() + 1));
    if (r) memcpy(r, s.c_str(), s.size() + 1);
    return r;
}

void sd_free(void* p) { free(p); }

}  // extern "C"
