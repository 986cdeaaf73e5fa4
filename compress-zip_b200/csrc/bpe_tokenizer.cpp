// bpe_tokenizer.cpp -- the .czm tokenizer on the host: tiktoken JSON loading,
// the pre-tokenizer of the shipped pattern as a hand-written scanner, byte-pair
// merging, special tokens, decoding, and a threaded batch encoder.
//
// Reference: rust/src/tiktoken.rs -- _byte_pair_merge (26-82), byte_pair_encode
// (84-107), CoreBPE::encode (215-268) with every special token allowed
// (encode_with_special_tokens, 498-501), decode_bytes (186-198), the JSON loader
// (505-563).  The reference pre-tokenizes with fancy-regex; the scanner below
// implements the one pattern kPattern alternative by alternative (leftmost
// match at each position, alternatives tried in order, possessive quantifiers
// never give characters back), with the Unicode 16.0 classes of
// unicode_classes.inc.
#include <algorithm>
#include <atomic>
#include <cctype>
#include <cstring>
#include <string>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <vector>

#include "czg_tok.h"

namespace {

#include "unicode_classes.inc"

const char kPattern[] =
    "'(?i:[sdmt]|ll|ve|re)|[^\\r\\n\\p{L}\\p{N}]?+\\p{L}++|\\p{N}{1,3}+| ?[^\\s\\p{L}\\p{N}]++[\\r\\n]*+"
    "|\\s++$|\\s*[\\r\\n]|\\s+(?!\\S)|\\s";

// ---- codepoint classes -------------------------------------------------------
enum : uint8_t { kL = 1, kN = 2, kS = 4 };

template <size_t K>
bool in_ranges(const uint32_t (&r)[K][2], uint32_t c) {
    size_t lo = 0, hi = K;   // first range with end >= c
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (r[mid][1] < c) lo = mid + 1; else hi = mid;
    }
    return lo < K && r[lo][0] <= c;
}

struct Classes {
    uint8_t low[256];
    Classes() {
        for (uint32_t c = 0; c < 256; c++) low[c] = slow(c);
    }
    static uint8_t slow(uint32_t c) {
        return (uint8_t)((in_ranges(kLetter, c) ? kL : 0) | (in_ranges(kNumber, c) ? kN : 0) |
                         (in_ranges(kSpace, c) ? kS : 0));
    }
    uint8_t operator()(uint32_t c) const { return c < 256 ? low[c] : slow(c); }
};
const Classes g_cls;

template <size_t K>
bool folds_to(const uint32_t (&f)[K], uint32_t c) {
    for (size_t i = 0; i < K; i++)
        if (f[i] == c) return true;
    return false;
}

// ---- UTF-8 -------------------------------------------------------------------
// Decodes valid UTF-8 (no overlongs, no surrogates, <= U+10FFFF) into codepoints
// and the byte offset of each; returns false on anything else.
bool decode_utf8(const uint8_t *s, size_t n, std::vector<uint32_t> &cp, std::vector<uint32_t> &off) {
    cp.clear();
    off.clear();
    size_t i = 0;
    while (i < n) {
        const uint8_t b = s[i];
        uint32_t c;
        size_t k;
        if (b < 0x80) { c = b; k = 1; }
        else if (b >= 0xC2 && b <= 0xDF) { c = b & 0x1F; k = 2; }
        else if (b >= 0xE0 && b <= 0xEF) { c = b & 0x0F; k = 3; }
        else if (b >= 0xF0 && b <= 0xF4) { c = b & 0x07; k = 4; }
        else return false;
        if (i + k > n) return false;
        for (size_t j = 1; j < k; j++) {
            if ((s[i + j] & 0xC0) != 0x80) return false;
            c = (c << 6) | (s[i + j] & 0x3F);
        }
        if ((k == 3 && (c < 0x800 || (c >= 0xD800 && c <= 0xDFFF))) || (k == 4 && (c < 0x10000 || c > 0x10FFFF)))
            return false;
        cp.push_back(c);
        off.push_back((uint32_t)i);
        i += k;
    }
    off.push_back((uint32_t)n);
    return true;
}

// ---- the pre-tokenizer -------------------------------------------------------
// Length (in codepoints, >= 1) of the match of kPattern starting at cp[i].
size_t match_at(const uint32_t *cp, size_t n, size_t i) {
    const uint32_t c0 = cp[i];
    // 1: '(?i:[sdmt]|ll|ve|re)
    if (c0 == '\'' && i + 1 < n) {
        const uint32_t c1 = cp[i + 1];
        if (folds_to(kFold_s, c1) || folds_to(kFold_d, c1) || folds_to(kFold_m, c1) || folds_to(kFold_t, c1))
            return 2;
        if (i + 2 < n) {
            const uint32_t c2 = cp[i + 2];
            if ((folds_to(kFold_l, c1) && folds_to(kFold_l, c2)) || (folds_to(kFold_v, c1) && folds_to(kFold_e, c2)) ||
                (folds_to(kFold_r, c1) && folds_to(kFold_e, c2)))
                return 3;
        }
    }
    const uint8_t k0 = g_cls(c0);
    // 2: [^\r\n\p{L}\p{N}]?+\p{L}++
    {
        size_t j = i;
        if (c0 != '\r' && c0 != '\n' && !(k0 & (kL | kN))) j++;
        size_t k = j;
        while (k < n && (g_cls(cp[k]) & kL)) k++;
        if (k > j) return k - i;
    }
    // 3: \p{N}{1,3}+
    if (k0 & kN) {
        size_t k = i + 1;
        while (k < n && k - i < 3 && (g_cls(cp[k]) & kN)) k++;
        return k - i;
    }
    // 4: ' ?[^\s\p{L}\p{N}]++[\r\n]*+'; without the space the class cannot start at a space
    {
        const size_t j = c0 == ' ' ? i + 1 : i;
        size_t k = j;
        while (k < n && !(g_cls(cp[k]) & (kL | kN | kS))) k++;
        if (k > j) {
            while (k < n && (cp[k] == '\r' || cp[k] == '\n')) k++;
            return k - i;
        }
    }
    if (!(k0 & kS)) return 1;   // unreachable: every non-space matched 2, 3 or 4
    size_t k = i + 1;           // the whitespace run [i, k)
    while (k < n && (g_cls(cp[k]) & kS)) k++;
    // 5: \s++$
    if (k == n) return k - i;
    // 6: \s*[\r\n] -- up to the last line break of the run
    for (size_t m = k; m > i; m--)
        if (cp[m - 1] == '\r' || cp[m - 1] == '\n') return m - i;
    // 7: \s+(?!\S) -- the run but its last character, which is followed by non-space
    if (k - i >= 2) return k - i - 1;
    // 8: \s
    return 1;
}

// ---- tokenizer ------------------------------------------------------------------
// bytes -> rank for tokens of at most 8 bytes (nearly every lookup): open addressing
// on the bytes packed into a 64-bit word and the length.
struct ShortRanks {
    struct Slot { uint64_t key; uint32_t rank; uint32_t len; };   // len 0: empty
    std::vector<Slot> slots;
    uint64_t mask = 0;
    static uint64_t pack(const uint8_t *p, size_t n) {
        uint64_t k = 0;
        memcpy(&k, p, n);
        return k;
    }
    static uint64_t hash(uint64_t k, size_t n) { return (k ^ (n * 0x9E3779B97F4A7C15ull)) * 0xD6E8FEB86659FD93ull; }
    void build(const std::vector<std::pair<std::string, uint32_t>> &items) {
        size_t cap = 16;
        while (cap < 4 * items.size()) cap <<= 1;
        slots.assign(cap, Slot{0, 0, 0});
        mask = cap - 1;
        for (const auto &it : items) {
            if (it.first.size() > 8 || it.first.empty()) continue;
            const uint64_t k = pack(reinterpret_cast<const uint8_t *>(it.first.data()), it.first.size());
            size_t h = (size_t)(hash(k, it.first.size()) >> 20) & mask;
            while (slots[h].len && !(slots[h].key == k && slots[h].len == it.first.size())) h = (h + 1) & mask;
            slots[h] = Slot{k, it.second, (uint32_t)it.first.size()};
        }
    }
    uint32_t find(const uint8_t *p, size_t n) const {   // n in 1..8
        const uint64_t k = pack(p, n);
        size_t h = (size_t)(hash(k, n) >> 20) & mask;
        for (;;) {
            const Slot &sl = slots[h];
            if (sl.len == 0) return UINT32_MAX;
            if (sl.key == k && sl.len == n) return sl.rank;
            h = (h + 1) & mask;
        }
    }
};

struct Tok {
    std::string store;                                   // every token's bytes, back to back
    std::unordered_map<std::string_view, uint32_t> rank;  // bytes -> rank (mergeable)
    ShortRanks short_rank;                               // the same for tokens of <= 8 bytes
    std::vector<std::pair<std::string, uint32_t>> specials;
    std::vector<std::pair<uint32_t, uint32_t>> dec;      // rank -> (offset, length) into store, or (~0, 0)
    std::string err;
    uint64_t id = 0;   // distinct per tokenizer ever created: keys the per-thread piece cache
    uint32_t find(const uint8_t *p, size_t n) const {
        if (n <= 8) return short_rank.find(p, n);
        auto it = rank.find(std::string_view(reinterpret_cast<const char *>(p), n));
        return it == rank.end() ? UINT32_MAX : it->second;
    }
};

// Per-thread memo of the merges of recent pieces (direct-mapped by a hash of the
// bytes; a slot keeps the last piece that landed on it).  Natural and synthetic
// text repeat their words, so most pieces skip the merge loop.
struct PieceCache {
    static constexpr size_t kSlots = 1 << 15, kMaxPiece = 48, kArena = 8 << 20;
    struct Slot { uint64_t h; uint32_t key_off, key_len, tok_off, tok_n; };
    std::vector<Slot> slots = std::vector<Slot>(kSlots, Slot{0, 0, 0, 0, 0});
    std::string keys;
    std::vector<uint32_t> toks;
    uint64_t owner = 0;   // the tokenizer whose merges these are
    void reset(uint64_t id) {
        keys.clear();
        toks.clear();
        std::fill(slots.begin(), slots.end(), Slot{0, 0, 0, 0, 0});
        owner = id;
    }
    static uint64_t hash(const uint8_t *p, size_t n) {
        uint64_t h = 0xCBF29CE484222325ull ^ n;
        for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 0x100000001B3ull;
        return h | 1;   // 0 marks an empty slot
    }
};
thread_local PieceCache t_cache;

// tiktoken.rs:26-82: the pair of adjacent parts with the lowest rank is merged until
// no adjacent pair is a token; ties go to the leftmost pair.
void byte_pair_encode(const Tok &t, const uint8_t *p, size_t n, std::vector<uint32_t> &out) {
    auto rank_of = [&](size_t a, size_t b) -> uint32_t { return t.find(p + a, b - a); };
    if (n == 1) {
        out.push_back(rank_of(0, 1));   // every byte is a token (checked at load)
        return;
    }
    struct Part { uint32_t start, rank; };
    std::vector<Part> parts(n + 1);
    for (size_t i = 0; i + 1 < n; i++) parts[i] = {(uint32_t)i, rank_of(i, i + 2)};
    parts[n - 1] = {(uint32_t)(n - 1), UINT32_MAX};
    parts[n] = {(uint32_t)n, UINT32_MAX};
    for (;;) {
        uint32_t best = UINT32_MAX;
        size_t bi = 0;
        for (size_t i = 0; i + 1 < parts.size(); i++)
            if (parts[i].rank < best) { best = parts[i].rank; bi = i; }
        if (best == UINT32_MAX) break;
        // the merged part [parts[bi].start, parts[bi + 2].start); new ranks of its pairs
        auto pair_rank = [&](size_t i) -> uint32_t {
            return i + 3 < parts.size() ? rank_of(parts[i].start, parts[i + 3].start) : UINT32_MAX;
        };
        if (bi > 0) parts[bi - 1].rank = pair_rank(bi - 1);
        parts[bi].rank = pair_rank(bi);
        parts.erase(parts.begin() + (ptrdiff_t)bi + 1);
    }
    for (size_t i = 0; i + 1 < parts.size(); i++) out.push_back(rank_of(parts[i].start, parts[i + 1].start));
}

// CoreBPE::encode with all specials allowed (tiktoken.rs:215-268)
bool encode_text(const Tok &t, const uint8_t *s, size_t n, std::vector<uint32_t> &out) {
    std::vector<uint32_t> cp, off;
    if (!decode_utf8(s, n, cp, off)) return false;
    const std::string_view text(reinterpret_cast<const char *>(s), n);
    size_t start = 0;   // byte offset
    size_t ci = 0;      // codepoint index of `start`
    for (;;) {
        // leftmost special token at or after start (the longest one on a tie)
        size_t sp = std::string_view::npos, sl = 0;
        uint32_t sr = 0;
        for (const auto &e : t.specials) {
            const size_t p = text.find(e.first, start);
            if (p != std::string_view::npos && (p < sp || (p == sp && e.first.size() > sl))) {
                sp = p;
                sl = e.first.size();
                sr = e.second;
            }
        }
        const size_t end = sp == std::string_view::npos ? n : sp;
        // codepoints of [start, end)
        size_t ce = ci;
        while (ce < cp.size() && off[ce] < end) ce++;
        for (size_t i = ci; i < ce;) {
            const size_t len = match_at(cp.data() + ci, ce - ci, i - ci);
            const uint32_t b0 = off[i], b1 = off[i + len];
            i += len;
            const uint32_t whole = t.find(s + b0, b1 - b0);
            if (whole != UINT32_MAX) {
                out.push_back(whole);
                continue;
            }
            const size_t pn = b1 - b0;
            if (pn > PieceCache::kMaxPiece) {
                byte_pair_encode(t, s + b0, pn, out);
                continue;
            }
            PieceCache &pc = t_cache;
            if (pc.owner != t.id) pc.reset(t.id);
            const uint64_t h = PieceCache::hash(s + b0, pn);
            PieceCache::Slot &sl = pc.slots[h & (PieceCache::kSlots - 1)];
            if (sl.h == h && sl.key_len == pn && memcmp(pc.keys.data() + sl.key_off, s + b0, pn) == 0) {
                out.insert(out.end(), pc.toks.begin() + sl.tok_off, pc.toks.begin() + sl.tok_off + sl.tok_n);
                continue;
            }
            const size_t o0 = out.size();
            byte_pair_encode(t, s + b0, pn, out);
            if (pc.keys.size() + pn > PieceCache::kArena || pc.toks.size() + (out.size() - o0) > PieceCache::kArena)
                pc.reset(t.id);
            sl = PieceCache::Slot{h, (uint32_t)pc.keys.size(), (uint32_t)pn, (uint32_t)pc.toks.size(),
                                  (uint32_t)(out.size() - o0)};
            pc.keys.append(reinterpret_cast<const char *>(s + b0), pn);
            pc.toks.insert(pc.toks.end(), out.begin() + o0, out.end());
        }
        if (sp == std::string_view::npos) break;
        out.push_back(sr);
        start = sp + sl;
        ci = ce;
        while (ci < cp.size() && off[ci] < start) ci++;
    }
    return true;
}

// ---- JSON ---------------------------------------------------------------------------
struct Json {
    const char *p, *e;
    bool ok = true;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool lit(char c) {
        ws();
        if (p < e && *p == c) { p++; return true; }
        return false;
    }
    static void put_utf8(std::string &s, uint32_t c) {
        if (c < 0x80) s += (char)c;
        else if (c < 0x800) { s += (char)(0xC0 | (c >> 6)); s += (char)(0x80 | (c & 0x3F)); }
        else if (c < 0x10000) {
            s += (char)(0xE0 | (c >> 12)); s += (char)(0x80 | ((c >> 6) & 0x3F)); s += (char)(0x80 | (c & 0x3F));
        } else {
            s += (char)(0xF0 | (c >> 18)); s += (char)(0x80 | ((c >> 12) & 0x3F));
            s += (char)(0x80 | ((c >> 6) & 0x3F)); s += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t &v) {
        if (e - p < 4) return false;
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    // a JSON string as UTF-8
    bool str(std::string &out) {
        out.clear();
        if (!lit('"')) return false;
        while (p < e && *p != '"') {
            if (*p != '\\') { out += *p++; continue; }
            if (++p >= e) return false;
            const char c = *p++;
            switch (c) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t v;
                    if (!hex4(v)) return false;
                    if (v >= 0xD800 && v <= 0xDBFF) {   // surrogate pair
                        uint32_t w;
                        if (e - p < 6 || p[0] != '\\' || p[1] != 'u') return false;
                        p += 2;
                        if (!hex4(w) || w < 0xDC00 || w > 0xDFFF) return false;
                        v = 0x10000 + ((v - 0xD800) << 10) + (w - 0xDC00);
                    } else if (v >= 0xDC00 && v <= 0xDFFF) {
                        return false;
                    }
                    put_utf8(out, v);
                    break;
                }
                default: return false;
            }
        }
        return lit('"');
    }
    bool uint(uint64_t &v) {
        ws();
        if (p >= e || *p < '0' || *p > '9') return false;
        v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            v = v * 10 + (uint64_t)(*p++ - '0');
            if (v > 0xFFFFFFFFull) return false;
        }
        return true;
    }
    bool skip() {   // any value
        ws();
        if (p >= e) return false;
        if (*p == '"') { std::string s; return str(s); }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            p++;
            if (lit(close)) return true;
            do {
                if (obj) { std::string k; if (!str(k) || !lit(':')) return false; }
                if (!skip()) return false;
            } while (lit(','));
            return lit(close);
        }
        const char *q = p;
        while (p < e && (std::isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) p++;
        return p > q;
    }
};

// the codepoints of a mergeable-rank key are its bytes (tiktoken.rs:517-527)
bool key_bytes(const std::string &utf8, std::string &out) {
    std::vector<uint32_t> cp, off;
    if (!decode_utf8(reinterpret_cast<const uint8_t *>(utf8.data()), utf8.size(), cp, off)) return false;
    out.clear();
    for (uint32_t c : cp) {
        if (c > 255) return false;
        out += (char)c;
    }
    return true;
}

int load(Tok &t, const char *json, size_t len) {
    Json j{json, json + len};
    std::string pat;
    bool have_pat = false, have_ranks = false;
    uint64_t explicit_n = 0;
    bool have_explicit = false;
    std::vector<std::pair<std::string, uint32_t>> ranks;
    if (!j.lit('{')) return CZG_TOK_E_JSON;
    if (!j.lit('}')) {
        do {
            std::string key;
            if (!j.str(key) || !j.lit(':')) return CZG_TOK_E_JSON;
            if (key == "pat_str") {
                if (!j.str(pat)) return CZG_TOK_E_JSON;
                have_pat = true;
            } else if (key == "mergeable_ranks" || key == "special_tokens") {
                const bool mr = key == "mergeable_ranks";
                if (!j.lit('{')) return CZG_TOK_E_JSON;
                if (!j.lit('}')) {
                    do {
                        std::string k, b;
                        uint64_t v;
                        if (!j.str(k) || !j.lit(':') || !j.uint(v)) return CZG_TOK_E_JSON;
                        if (mr) {
                            if (!key_bytes(k, b)) { t.err = "mergeable key outside bytes 0..255"; return CZG_TOK_E_VOCAB; }
                            ranks.emplace_back(b, (uint32_t)v);
                        } else {
                            t.specials.emplace_back(k, (uint32_t)v);
                        }
                    } while (j.lit(','));
                    if (!j.lit('}')) return CZG_TOK_E_JSON;
                }
                if (mr) have_ranks = true;
            } else if (key == "explicit_n_vocab") {
                j.ws();
                if (j.p < j.e && *j.p == 'n') {
                    if (!j.skip()) return CZG_TOK_E_JSON;
                } else {
                    if (!j.uint(explicit_n)) return CZG_TOK_E_JSON;
                    have_explicit = true;
                }
            } else if (!j.skip()) {
                return CZG_TOK_E_JSON;
            }
        } while (j.lit(','));
        if (!j.lit('}')) return CZG_TOK_E_JSON;
    }
    if (!have_pat || !have_ranks) { t.err = "pat_str or mergeable_ranks missing"; return CZG_TOK_E_JSON; }
    if (pat != kPattern) { t.err = "unsupported pre-tokenizer pattern"; return CZG_TOK_E_PATTERN; }
    // duplicate keys: the last one wins, as in a JSON map
    std::unordered_map<std::string, uint32_t> uniq;
    for (auto &r : ranks) uniq[r.first] = r.second;
    std::unordered_map<std::string, uint32_t> uspec;
    for (auto &s : t.specials) uspec[s.first] = s.second;
    t.specials.assign(uspec.begin(), uspec.end());
    if (have_explicit && explicit_n != uniq.size() + t.specials.size()) {   // tiktoken.rs:556-560
        t.err = "explicit_n_vocab != computed size";
        return CZG_TOK_E_VOCAB;
    }
    size_t total = 0;
    uint32_t max_rank = 0;
    for (auto &r : uniq) { total += r.first.size(); max_rank = std::max(max_rank, r.second); }
    for (auto &s : t.specials) max_rank = std::max(max_rank, s.second);
    t.store.reserve(total);
    std::vector<std::pair<size_t, size_t>> where;
    for (auto &r : uniq) { where.emplace_back(t.store.size(), r.first.size()); t.store += r.first; }
    t.dec.assign((size_t)max_rank + 1, {UINT32_MAX, 0});
    size_t i = 0;
    for (auto &r : uniq) {
        const std::string_view v(t.store.data() + where[i].first, where[i].second);
        t.rank[v] = r.second;
        t.dec[r.second] = {(uint32_t)where[i].first, (uint32_t)where[i].second};
        i++;
    }
    t.short_rank.build(std::vector<std::pair<std::string, uint32_t>>(uniq.begin(), uniq.end()));
    for (int b = 0; b < 256; b++) {
        const uint8_t c = (uint8_t)b;
        if (t.find(&c, 1) == UINT32_MAX) {
            t.err = "a byte has no token";
            return CZG_TOK_E_VOCAB;
        }
    }
    return CZG_TOK_OK;
}

}  // namespace

struct czg_tok {
    Tok t;
    mutable std::string last_error;
};

extern "C" {

const char *czg_tok_pattern(void) { return kPattern; }

int czg_tok_create(const char *json, size_t json_len, czg_tok **out) {
    if (!json || !out) return CZG_TOK_E_ARG;
    *out = nullptr;
    static std::atomic<uint64_t> next_id{1};
    czg_tok *h = new czg_tok();
    h->t.id = next_id.fetch_add(1);
    const int st = load(h->t, json, json_len);
    if (st != CZG_TOK_OK) {
        delete h;
        return st;
    }
    *out = h;
    return CZG_TOK_OK;
}

void czg_tok_destroy(czg_tok *tok) { delete tok; }

const char *czg_tok_last_error(const czg_tok *tok) { return tok ? tok->last_error.c_str() : ""; }

int czg_tok_encode(const czg_tok *tok, const char *text, size_t len, uint32_t *out, size_t cap, size_t *n_out) {
    if (!tok || (!text && len) || !n_out) return CZG_TOK_E_ARG;
    std::vector<uint32_t> ids;
    ids.reserve(len / 2 + 16);
    if (!encode_text(tok->t, reinterpret_cast<const uint8_t *>(text), len, ids)) {
        tok->last_error = "input is not valid UTF-8";
        return CZG_TOK_E_UTF8;
    }
    *n_out = ids.size();
    if (!out || ids.size() > cap) return out ? CZG_TOK_E_CAPACITY : CZG_TOK_OK;
    if (!ids.empty()) memcpy(out, ids.data(), ids.size() * 4);
    return CZG_TOK_OK;
}

int czg_tok_encode_batch(const czg_tok *tok, size_t n_docs, const char *const *texts, const size_t *lens,
                         uint32_t *out, const size_t *out_offsets, size_t *n_out, int threads) {
    if (!tok || (n_docs && (!texts || !lens || !out || !out_offsets || !n_out))) return CZG_TOK_E_ARG;
    int nt = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
    nt = (int)std::min<size_t>((size_t)nt, std::max<size_t>(n_docs, 1));
    std::atomic<size_t> next{0};
    std::atomic<int> status{CZG_TOK_OK};
    auto work = [&]() {
        std::vector<uint32_t> ids;
        for (;;) {
            const size_t i = next.fetch_add(1);
            if (i >= n_docs) break;
            ids.clear();
            if (!encode_text(tok->t, reinterpret_cast<const uint8_t *>(texts[i]), lens[i], ids)) {
                status.store(CZG_TOK_E_UTF8);
                n_out[i] = 0;
                continue;
            }
            n_out[i] = ids.size();   // <= lens[i]: every token has at least one byte
            if (!ids.empty()) memcpy(out + out_offsets[i], ids.data(), ids.size() * 4);
        }
    };
    std::vector<std::thread> pool;
    for (int k = 1; k < nt; k++) pool.emplace_back(work);
    work();
    for (auto &th : pool) th.join();
    if (status.load() != CZG_TOK_OK) tok->last_error = "a document is not valid UTF-8";
    return status.load();
}

int czg_tok_decode(const czg_tok *tok, const uint32_t *ids, size_t n, uint8_t *out, size_t cap, size_t *n_out) {
    if (!tok || (!ids && n) || !n_out) return CZG_TOK_E_ARG;
    const Tok &t = tok->t;
    size_t need = 0;
    for (size_t i = 0; i < n; i++) {
        const uint32_t id = ids[i];
        if (id < t.dec.size() && t.dec[id].first != UINT32_MAX) { need += t.dec[id].second; continue; }
        bool found = false;
        for (const auto &s : t.specials)
            if (s.second == id) { need += s.first.size(); found = true; break; }
        if (!found) {
            tok->last_error = "Invalid token for decoding: " + std::to_string(id);
            return CZG_TOK_E_TOKEN;
        }
    }
    *n_out = need;
    if (!out || need > cap) return out ? CZG_TOK_E_CAPACITY : CZG_TOK_OK;
    size_t o = 0;
    for (size_t i = 0; i < n; i++) {
        const uint32_t id = ids[i];
        if (id < t.dec.size() && t.dec[id].first != UINT32_MAX) {
            memcpy(out + o, t.store.data() + t.dec[id].first, t.dec[id].second);
            o += t.dec[id].second;
            continue;
        }
        for (const auto &s : t.specials)
            if (s.second == id) { memcpy(out + o, s.first.data(), s.first.size()); o += s.first.size(); break; }
    }
    return CZG_TOK_OK;
}

}  // extern "C"
