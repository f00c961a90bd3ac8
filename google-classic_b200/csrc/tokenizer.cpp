// tokenizer.cpp -- the reference's greedy longest-match tokenizer
// (llm_tokenize, src/ai/llm.c:178-221) with the same output, host side.
//
// The reference scans the whole vocabulary at every text position (strlen +
// strncmp per token: O(text bytes x vocab x token length), tens of
// milliseconds for a few hundred bytes on a 32k vocabulary), and scans it
// again for the byte fallback (find_byte_token, llm.c:150-175).  Here the
// vocabulary becomes a byte trie once, at creation:
//   * each node that ends a token string holds the smallest vocabulary index
//     with that string -- the reference keeps the first token of the longest
//     matching length (strictly longer replaces), and two tokens of the same
//     length that both match at a position are the same string;
//   * children sit in one flat edge array per node, sorted by byte (binary
//     search), the root's in a 256-entry table;
//   * the byte fallback of every byte value is resolved once, in the
//     reference's order: the first "<0xNN>" token (upper-case hex), else the
//     first token equal to the byte's GPT-2 byte-level string as the
//     reference builds it (init_byte_to_unicode, llm.c:116-147), else unk.
// Tokenizing walks the trie from each position for at most the longest
// token's length: O(text bytes x longest token).
#include "holo_b200.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <utility>
#include <vector>

struct holo_tokenizer {
    // node 0 is the root; node n's children are edges [first[n], first[n+1])
    std::vector<uint32_t> first;
    std::vector<uint8_t> edge_byte;
    std::vector<int32_t> edge_node;
    std::vector<int32_t> token;   // smallest vocabulary index ending here, or -1
    int32_t root_child[256];
    int32_t fallback[256];
    int bos, unk;
};

namespace {

// The byte-level strings of the reference's byte map: bytes 33..126 stand for
// themselves; every other byte, in increasing order, takes the next code point
// from U+0100 on, except bytes 161 and 166..172, which have no string (the
// reference skips them, so they fall through to unk).  UTF-8, two bytes.
std::string byte_level_string(int b) {
    if (b >= 33 && b <= 126) return std::string(1, (char)b);
    if (b == 161 || (b >= 166 && b <= 172)) return std::string();
    int n = 0;
    for (int i = 0; i < b; ++i) {
        if (i >= 33 && i <= 126) continue;
        if (i == 161 || (i >= 166 && i <= 172)) continue;
        ++n;
    }
    const int cp = 256 + n;   // < 0x800 for every byte
    std::string s;
    s.push_back((char)(0xC0 | (cp >> 6)));
    s.push_back((char)(0x80 | (cp & 0x3F)));
    return s;
}

int32_t child_of(const holo_tokenizer *t, int32_t node, uint8_t c) {
    if (node == 0) return t->root_child[c];
    const uint8_t *b = t->edge_byte.data();
    uint32_t lo = t->first[node], hi = t->first[node + 1];
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (b[mid] < c) lo = mid + 1;
        else hi = mid;
    }
    return (lo < t->first[node + 1] && b[lo] == c) ? t->edge_node[lo] : -1;
}

// smallest index of a vocabulary string equal to s, or -1
int32_t exact(const holo_tokenizer *t, const std::string &s) {
    if (s.empty()) return -1;
    int32_t node = 0;
    for (unsigned char c : s) {
        node = child_of(t, node, c);
        if (node < 0) return -1;
    }
    return t->token[node];
}

}  // namespace

extern "C" holo_tokenizer *holo_tokenizer_create(const char *const *vocab, int vocab_size, int bos_token,
                                                 int unk_token) {
    if (vocab_size < 0 || (vocab_size > 0 && !vocab)) return nullptr;
    holo_tokenizer *t = new (std::nothrow) holo_tokenizer;
    if (!t) return nullptr;
    try {
        t->bos = bos_token;
        t->unk = unk_token;
        // (string, index) of every non-empty token, sorted by bytes then index:
        // equal strings become one trie path holding the first index
        std::vector<std::pair<const char *, int>> ent;
        ent.reserve((size_t)vocab_size);
        size_t total = 0;   // trie nodes <= total string bytes + 1: node ids must fit int32
        for (int i = 0; i < vocab_size; ++i)
            if (vocab[i] && vocab[i][0]) {
                ent.emplace_back(vocab[i], i);
                total += std::strlen(vocab[i]);
            }
        if (total >= (size_t)INT32_MAX) {
            delete t;
            return nullptr;
        }
        std::stable_sort(ent.begin(), ent.end(), [](const std::pair<const char *, int> &a,
                                                    const std::pair<const char *, int> &b) {
            return std::strcmp(a.first, b.first) < 0;   // strcmp orders bytes as unsigned char
        });
        // Depth-first construction over the sorted strings: the path of the
        // previous string is the stack; each string shares its common prefix
        // with it and appends new nodes.  Children of a node are created in
        // increasing byte order, so the per-node edge lists come out sorted.
        std::vector<int32_t> parent{-1};
        std::vector<uint8_t> via{0};
        t->token.assign(1, -1);
        std::vector<int32_t> path{0};   // path[d] = node at depth d of the previous string
        const char *prev = "";
        for (const auto &e : ent) {
            const unsigned char *s = reinterpret_cast<const unsigned char *>(e.first);
            const unsigned char *p = reinterpret_cast<const unsigned char *>(prev);
            size_t common = 0;
            while (s[common] && s[common] == p[common]) ++common;
            path.resize(common + 1);
            for (size_t d = common; s[d]; ++d) {
                parent.push_back(path.back());
                via.push_back(s[d]);
                t->token.push_back(-1);
                path.push_back((int32_t)t->token.size() - 1);
            }
            if (t->token[path.back()] < 0) t->token[path.back()] = e.second;   // first index of the string
            prev = e.first;
        }
        // flatten: children grouped by parent, in creation (= byte) order
        const size_t nn = t->token.size();
        std::vector<uint32_t> count(nn + 1, 0);
        for (size_t n = 1; n < nn; ++n) count[parent[n]]++;
        t->first.assign(nn + 1, 0);
        for (size_t n = 0; n < nn; ++n) t->first[n + 1] = t->first[n] + count[n];
        t->edge_byte.resize(nn ? nn - 1 : 0);
        t->edge_node.resize(nn ? nn - 1 : 0);
        std::vector<uint32_t> fill(t->first.begin(), t->first.end() - 1);
        for (size_t n = 1; n < nn; ++n) {
            const uint32_t k = fill[parent[n]]++;
            t->edge_byte[k] = via[n];
            t->edge_node[k] = (int32_t)n;
        }
        for (int c = 0; c < 256; ++c) t->root_child[c] = -1;
        for (uint32_t k = t->first[0]; k < t->first[1]; ++k) t->root_child[t->edge_byte[k]] = t->edge_node[k];
        // byte fallback, resolved once per byte value
        for (int b = 0; b < 256; ++b) {
            char hex[8];
            std::snprintf(hex, sizeof hex, "<0x%02X>", b);
            int32_t id = exact(t, hex);
            if (id < 0) id = exact(t, byte_level_string(b));
            t->fallback[b] = id >= 0 ? id : unk_token;
        }
    } catch (...) {
        delete t;
        return nullptr;
    }
    return t;
}

extern "C" int holo_tokenize(const holo_tokenizer *t, const char *text, int *tokens, int max_tokens, int add_bos) {
    if (!t || !text || (max_tokens > 0 && !tokens)) return -1;
    int n = 0;
    if (add_bos && n < max_tokens) tokens[n++] = t->bos;
    const unsigned char *p = reinterpret_cast<const unsigned char *>(text);
    while (*p && n < max_tokens) {
        int32_t node = 0, best = -1;
        size_t best_len = 0;
        for (size_t d = 0; p[d]; ++d) {
            node = child_of(t, node, p[d]);
            if (node < 0) break;
            if (t->token[node] >= 0) {
                best = t->token[node];
                best_len = d + 1;
            }
        }
        if (best_len) {
            tokens[n++] = best;
            p += best_len;
        } else {
            tokens[n++] = t->fallback[*p];
            ++p;
        }
    }
    return n;
}

extern "C" void holo_tokenizer_free(holo_tokenizer *t) { delete t; }
