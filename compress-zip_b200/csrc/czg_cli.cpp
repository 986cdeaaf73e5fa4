// czg_cli.cpp -- the compress / decompress command line of the reference
// (rust/src/main.rs:18-74) as one native program: model and tokenizer loading
// (main.rs:124-175), the native BPE tokenizer (libczg_tok.so), the chunk loops on
// the GPU through the C ABI (libczg.so, in place of main.rs:206-238 / 377-396),
// the CZIPv1 container (rust/src/file_format.rs), the outer codec (brotli q11 /
// lgwin 22 or zstd 22 from the system libraries, main.rs:259-281), and the
// detokenised, lossily decoded UTF-8 output (main.rs:401-412).
//
//   czg-cli compress   -m MODEL.czm -i in.txt  -o out.czip [-t tok.json] [-c brotli|zstd] [-L 1..5]
//   czg-cli decompress -m MODEL.czm -i in.czip -o out.txt  [-t tok.json]
//   czg-cli selftest   (host parts only: MD5, container, codecs; no GPU)
//   czg-cli outer zstd|brotli compress|decompress IN OUT   (the outer codec alone)
//   czg-cli md5-path PATH   (the model_id_hash of a model path, hex)
//
// The outer codec libraries are loaded at run time (dlopen) and driven with the
// same streaming calls as compress_zip_b200/outer_codec.py, so both front ends
// write identical files.
#include <dlfcn.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "czg.h"
#include "czg_tok.h"
#include "czm_parse.h"

namespace {

using Bytes = std::vector<uint8_t>;

[[noreturn]] void die(const std::string &m) { throw std::runtime_error(m); }

Bytes read_file(const std::string &p) {
    std::ifstream f(p, std::ios::binary);
    if (!f) die("cannot open " + p);
    std::ostringstream ss;
    ss << f.rdbuf();
    const std::string s = ss.str();
    return Bytes(s.begin(), s.end());
}

void write_file(const std::string &p, const uint8_t *d, size_t n, const uint8_t *d2 = nullptr, size_t n2 = 0) {
    std::ofstream f(p, std::ios::binary);
    if (!f) die("cannot create " + p);
    f.write(reinterpret_cast<const char *>(d), (std::streamsize)n);
    if (d2) f.write(reinterpret_cast<const char *>(d2), (std::streamsize)n2);
    if (!f) die("cannot write " + p);
}

// ---- MD5 (RFC 1321), for model_id_hash = md5(model path)[:8] (main.rs:79-85) ----
struct Md5 {
    uint32_t K[64];
    Md5() {
        for (int i = 0; i < 64; i++) K[i] = (uint32_t)(std::fabs(std::sin((double)(i + 1))) * 4294967296.0);
    }
    static uint32_t rol(uint32_t x, int c) { return (x << c) | (x >> (32 - c)); }
    std::string hex(const uint8_t *msg, size_t len) const {
        static const int S[64] = {7, 12, 17, 22, 7, 12, 17, 22, 7, 12, 17, 22, 7, 12, 17, 22,
                                  5, 9,  14, 20, 5, 9,  14, 20, 5, 9,  14, 20, 5, 9,  14, 20,
                                  4, 11, 16, 23, 4, 11, 16, 23, 4, 11, 16, 23, 4, 11, 16, 23,
                                  6, 10, 15, 21, 6, 10, 15, 21, 6, 10, 15, 21, 6, 10, 15, 21};
        Bytes m(msg, msg + len);
        m.push_back(0x80);
        while (m.size() % 64 != 56) m.push_back(0);
        const uint64_t bits = (uint64_t)len * 8;
        for (int i = 0; i < 8; i++) m.push_back((uint8_t)(bits >> (8 * i)));
        uint32_t a0 = 0x67452301, b0 = 0xefcdab89, c0 = 0x98badcfe, d0 = 0x10325476;
        for (size_t off = 0; off < m.size(); off += 64) {
            uint32_t w[16];
            for (int i = 0; i < 16; i++)
                w[i] = (uint32_t)m[off + 4 * i] | ((uint32_t)m[off + 4 * i + 1] << 8) |
                       ((uint32_t)m[off + 4 * i + 2] << 16) | ((uint32_t)m[off + 4 * i + 3] << 24);
            uint32_t A = a0, B = b0, C = c0, D = d0;
            for (int i = 0; i < 64; i++) {
                uint32_t F;
                int g;
                if (i < 16) { F = (B & C) | (~B & D); g = i; }
                else if (i < 32) { F = (D & B) | (~D & C); g = (5 * i + 1) % 16; }
                else if (i < 48) { F = B ^ C ^ D; g = (3 * i + 5) % 16; }
                else { F = C ^ (B | ~D); g = (7 * i) % 16; }
                F = F + A + K[i] + w[g];
                A = D;
                D = C;
                C = B;
                B = B + rol(F, S[i]);
            }
            a0 += A; b0 += B; c0 += C; d0 += D;
        }
        char out[33];
        const uint32_t v[4] = {a0, b0, c0, d0};
        for (int i = 0; i < 16; i++) snprintf(out + 2 * i, 3, "%02x", (v[i / 4] >> (8 * (i % 4))) & 0xFF);
        return std::string(out, 32);
    }
};

uint32_t hash_model_path(const std::string &path) {
    return (uint32_t)std::stoul(Md5().hex(reinterpret_cast<const uint8_t *>(path.data()), path.size()).substr(0, 8),
                                nullptr, 16);
}

// ---- outer codec: the system zstd / brotli libraries, loaded at run time ----
void *load_lib(const char *a, const char *b) {
    void *h = dlopen(a, RTLD_NOW);
    if (!h) h = dlopen(b, RTLD_NOW);
    if (!h) die(std::string("cannot load ") + a);
    return h;
}
template <class F>
F sym(void *lib, const char *name) {
    void *p = dlsym(lib, name);
    if (!p) die(std::string("missing symbol ") + name);
    return reinterpret_cast<F>(p);
}

struct ZBufIn { const void *src; size_t size, pos; };
struct ZBufOut { void *dst; size_t size, pos; };

Bytes zstd_compress(const Bytes &in, int level) {
    void *L = load_lib("libzstd.so.1", "libzstd.so");
    auto create = sym<void *(*)()>(L, "ZSTD_createCCtx");
    auto freec = sym<size_t (*)(void *)>(L, "ZSTD_freeCCtx");
    auto setp = sym<size_t (*)(void *, int, int)>(L, "ZSTD_CCtx_setParameter");
    auto stream2 = sym<size_t (*)(void *, ZBufOut *, ZBufIn *, int)>(L, "ZSTD_compressStream2");
    auto outsize = sym<size_t (*)()>(L, "ZSTD_CStreamOutSize");
    auto iserr = sym<unsigned (*)(size_t)>(L, "ZSTD_isError");
    void *cctx = create();
    setp(cctx, 100, level);   // ZSTD_c_compressionLevel
    ZBufIn ib{in.data(), in.size(), 0};
    const size_t cap = outsize();
    Bytes buf(cap), out;
    for (;;) {
        ZBufOut ob{buf.data(), cap, 0};
        const int mode = ib.pos < ib.size ? 0 : 2;   // ZSTD_e_continue, then ZSTD_e_end
        const size_t r = stream2(cctx, &ob, &ib, mode);
        if (iserr(r)) { freec(cctx); die("zstd compression failed"); }
        out.insert(out.end(), buf.begin(), buf.begin() + (ptrdiff_t)ob.pos);
        if (mode == 2 && r == 0) break;
    }
    freec(cctx);
    return out;
}

Bytes zstd_decompress(const Bytes &in, size_t off) {
    void *L = load_lib("libzstd.so.1", "libzstd.so");
    auto create = sym<void *(*)()>(L, "ZSTD_createDCtx");
    auto freed = sym<size_t (*)(void *)>(L, "ZSTD_freeDCtx");
    auto dstream = sym<size_t (*)(void *, ZBufOut *, ZBufIn *)>(L, "ZSTD_decompressStream");
    auto outsize = sym<size_t (*)()>(L, "ZSTD_DStreamOutSize");
    auto iserr = sym<unsigned (*)(size_t)>(L, "ZSTD_isError");
    void *d = create();
    ZBufIn ib{in.data() + off, in.size() - off, 0};
    const size_t cap = outsize();
    Bytes buf(cap), out;
    for (;;) {
        ZBufOut ob{buf.data(), cap, 0};
        const size_t r = dstream(d, &ob, &ib);
        if (iserr(r)) { freed(d); die("zstd: corrupt stream"); }
        out.insert(out.end(), buf.begin(), buf.begin() + (ptrdiff_t)ob.pos);
        if (ib.pos >= ib.size && ob.pos < cap) {
            freed(d);
            if (r != 0) die("zstd: truncated frame");
            return out;
        }
    }
}

Bytes brotli_compress(const Bytes &in, int quality, int lgwin) {
    void *L = load_lib("libbrotlienc.so.1", "libbrotlienc.so");
    auto create = sym<void *(*)(void *, void *, void *)>(L, "BrotliEncoderCreateInstance");
    auto setp = sym<int (*)(void *, int, uint32_t)>(L, "BrotliEncoderSetParameter");
    auto stream = sym<int (*)(void *, int, size_t *, const uint8_t **, size_t *, uint8_t **, size_t *)>(
        L, "BrotliEncoderCompressStream");
    auto finished = sym<int (*)(void *)>(L, "BrotliEncoderIsFinished");
    auto destroy = sym<void (*)(void *)>(L, "BrotliEncoderDestroyInstance");
    void *st = create(nullptr, nullptr, nullptr);
    setp(st, 1, (uint32_t)quality);   // BROTLI_PARAM_QUALITY
    setp(st, 2, (uint32_t)lgwin);     // BROTLI_PARAM_LGWIN
    size_t avail_in = in.size();
    const uint8_t *next_in = in.data();
    const size_t cap = 4096;
    Bytes buf(cap), out;
    int op = 0;   // BROTLI_OPERATION_PROCESS until all input is taken, then FINISH
    for (;;) {
        if (op == 0 && avail_in == 0) op = 2;
        size_t avail_out = cap;
        uint8_t *next_out = buf.data();
        if (!stream(st, op, &avail_in, &next_in, &avail_out, &next_out, nullptr)) {
            destroy(st);
            die("brotli encoder error");
        }
        out.insert(out.end(), buf.begin(), buf.begin() + (ptrdiff_t)(cap - avail_out));
        if (op == 2 && finished(st)) break;
    }
    destroy(st);
    return out;
}

Bytes brotli_decompress(const Bytes &in, size_t off) {
    void *L = load_lib("libbrotlidec.so.1", "libbrotlidec.so");
    auto create = sym<void *(*)(void *, void *, void *)>(L, "BrotliDecoderCreateInstance");
    auto stream = sym<int (*)(void *, size_t *, const uint8_t **, size_t *, uint8_t **, size_t *)>(
        L, "BrotliDecoderDecompressStream");
    auto destroy = sym<void (*)(void *)>(L, "BrotliDecoderDestroyInstance");
    void *st = create(nullptr, nullptr, nullptr);
    size_t avail_in = in.size() - off;
    const uint8_t *next_in = in.data() + off;
    const size_t cap = 1 << 16;
    Bytes buf(cap), out;
    for (;;) {
        size_t avail_out = cap;
        uint8_t *next_out = buf.data();
        const int r = stream(st, &avail_in, &next_in, &avail_out, &next_out, nullptr);
        out.insert(out.end(), buf.begin(), buf.begin() + (ptrdiff_t)(cap - avail_out));
        if (r == 1) { destroy(st); return out; }   // BROTLI_DECODER_RESULT_SUCCESS
        if (r == 3) continue;                       // NEEDS_MORE_OUTPUT
        destroy(st);
        die("brotli: corrupt or truncated stream");
    }
}

enum { kZstd = 0, kBrotli = 1 };

Bytes outer_compress(const Bytes &in, int codec) {
    return codec == kZstd ? zstd_compress(in, 22) : brotli_compress(in, 11, 22);
}
Bytes outer_decompress(const Bytes &in, size_t off, int codec) {
    return codec == kZstd ? zstd_decompress(in, off) : brotli_decompress(in, off);
}

// ---- CZIPv1 container (rust/src/file_format.rs) ----
//  outer (16 B, file_format.rs:77-154): "CZIPv1", flags u8, codec u8, uncompressed_len u32,
//  header_len u32; payload = codec(inner header || chunk bytes); inner (file_format.rs:158-257):
//  model_id_hash u32, chunk_count u32, last_chunk_tokens u16, tokenizer_id u8,
//  context_length_log2 u8 (0 reads as 6), chunk_count x u16 byte lengths.
void put_u16(Bytes &b, uint32_t v) { b.push_back((uint8_t)v); b.push_back((uint8_t)(v >> 8)); }
void put_u32(Bytes &b, uint32_t v) { for (int i = 0; i < 4; i++) b.push_back((uint8_t)(v >> (8 * i))); }
uint32_t get_u16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
uint32_t get_u32(const uint8_t *p) { return get_u16(p) | (get_u16(p + 2) << 16); }

struct Container {
    int codec = kBrotli;
    uint32_t flags = 0, uncompressed_len = 0, model_id_hash = 0, last_chunk_tokens = 0;
    uint32_t tokenizer_id = 0, log2 = 6;
    std::vector<uint32_t> lens;
    Bytes data;   // chunk bytes back to back

    uint32_t tokens_per_chunk() const { return (1u << log2) & 0xFFFF; }
    uint32_t chunk_tokens(size_t i) const { return i + 1 == lens.size() ? last_chunk_tokens : tokens_per_chunk(); }
    void outer(Bytes &o) const {
        const char *magic = "CZIPv1";
        o.assign(magic, magic + 6);
        o.push_back((uint8_t)flags);
        o.push_back((uint8_t)codec);
        put_u32(o, uncompressed_len);
        put_u32(o, (uint32_t)(12 + 2 * lens.size()));
    }
    Bytes payload() const {
        Bytes p;
        put_u32(p, model_id_hash);
        put_u32(p, (uint32_t)lens.size());
        put_u16(p, last_chunk_tokens);
        p.push_back((uint8_t)tokenizer_id);
        p.push_back((uint8_t)log2);
        for (uint32_t l : lens) put_u16(p, l);
        p.insert(p.end(), data.begin(), data.end());
        return p;
    }
    static Container parse(const Bytes &file, Bytes &payload_out) {
        if (file.size() < 16) die("Outer header too short");
        if (memcmp(file.data(), "CZIPv1", 6) != 0) die("Invalid magic bytes");
        Container c;
        c.flags = file[6];
        c.codec = file[7];
        if (c.codec != kZstd && c.codec != kBrotli) die("Unknown codec: " + std::to_string(c.codec));
        c.uncompressed_len = get_u32(&file[8]);
        payload_out = outer_decompress(file, 16, c.codec);
        const Bytes &p = payload_out;
        if (p.size() < 12) die("Inner header too short");
        c.model_id_hash = get_u32(&p[0]);
        const uint32_t cc = get_u32(&p[4]);
        c.last_chunk_tokens = get_u16(&p[8]);
        c.tokenizer_id = p[10];
        c.log2 = p[11] ? p[11] : 6;
        if (p.size() < 12 + 2 * (size_t)cc) die("Inner header too short for " + std::to_string(cc) + " chunks");
        size_t off = 12 + 2 * (size_t)cc, total = 0;
        for (uint32_t i = 0; i < cc; i++) {
            c.lens.push_back(get_u16(&p[12 + 2 * i]));
            total += c.lens.back();
        }
        if (p.size() < off + total) die("Chunk data truncated");
        c.data.assign(p.begin() + (ptrdiff_t)off, p.begin() + (ptrdiff_t)(off + total));
        return c;
    }
};

// ---- UTF-8: lossy decoding like String::from_utf8_lossy (one U+FFFD per maximal ill-formed subpart) ----
std::string utf8_lossy(const uint8_t *s, size_t n) {
    std::string out;
    out.reserve(n);
    size_t i = 0;
    while (i < n) {
        const uint8_t b = s[i];
        if (b < 0x80) { out += (char)b; i++; continue; }
        size_t need = 0;
        uint8_t lo = 0x80, hi = 0xBF;
        if (b >= 0xC2 && b <= 0xDF) need = 1;
        else if (b >= 0xE0 && b <= 0xEF) { need = 2; if (b == 0xE0) lo = 0xA0; if (b == 0xED) hi = 0x9F; }
        else if (b >= 0xF0 && b <= 0xF4) { need = 3; if (b == 0xF0) lo = 0x90; if (b == 0xF4) hi = 0x8F; }
        size_t k = 1;
        bool ok = need > 0;
        for (; ok && k <= need; k++) {
            if (i + k >= n) { ok = false; break; }
            const uint8_t c = s[i + k];
            if (c < (k == 1 ? lo : 0x80) || c > (k == 1 ? hi : 0xBF)) { ok = false; break; }
        }
        if (ok) {
            out.append(reinterpret_cast<const char *>(s + i), need + 1);
            i += need + 1;
        } else {
            out += "\xEF\xBF\xBD";
            i += std::max<size_t>(1, k);   // the valid prefix of the sequence is one subpart
        }
    }
    return out;
}

// ---- model, tokenizer, engine ----
struct Loaded {
    Bytes model;
    czg::CzmFile czm;
    czg_tok *tok = nullptr;
    czg_ctx *ctx = nullptr;
    int context_length = 64;
    ~Loaded() {
        if (tok) czg_tok_destroy(tok);
        if (ctx) czg_ctx_destroy(ctx);
    }
};

void load(Loaded &L, const std::string &model_path, const std::string &tok_path, int device) {
    printf("Loading model from '%s'...\n", model_path.c_str());
    L.model = read_file(model_path);
    const std::string err = czg::parse_czm(L.model.data(), L.model.size(), L.czm);
    if (!err.empty()) die("Failed to load model: " + err);
    auto it = L.czm.metadata.find("context_length");
    if (it != L.czm.metadata.end()) L.context_length = std::stoi(it->second);
    Bytes json;
    if (!tok_path.empty()) {
        printf("Loading tokenizer from '%s'...\n", tok_path.c_str());
        json = read_file(tok_path);
    } else {
        printf("Loading embedded tokenizer from model...\n");
        auto t = L.czm.tensors.find("tokenizer.data");
        if (t == L.czm.tensors.end()) die("model has no embedded tokenizer (tokenizer.data)");
        Bytes packed(t->second.data, t->second.data + t->second.nbytes);
        auto c = L.czm.metadata.find("tokenizer_codec");
        const std::string codec = c == L.czm.metadata.end() ? "zstd" : c->second;
        if (codec == "zstd") json = zstd_decompress(packed, 0);
        else if (codec == "brotli") json = brotli_decompress(packed, 0);
        else die("Unknown tokenizer codec: " + codec);
    }
    const int st = czg_tok_create(reinterpret_cast<const char *>(json.data()), json.size(), &L.tok);
    if (st != CZG_TOK_OK) die("tokenizer: status " + std::to_string(st));
    if (czg_ctx_create(device, L.model.data(), L.model.size(), &L.ctx) != 0)
        die(std::string("engine: ") + czg_last_error(nullptr));
}

double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int do_compress(const std::string &model, const std::string &tokp, const std::string &in, const std::string &out,
                const std::string &codec_str, int level) {
    const double t0 = now();
    int codec;
    if (codec_str == "brotli") codec = kBrotli;
    else if (codec_str == "zstd") codec = kZstd;
    else die("Unknown codec: " + codec_str);
    Loaded L;
    load(L, model, tokp, 0);
    printf("Reading input from '%s'...\n", in.c_str());
    const Bytes text = read_file(in);
    printf("Tokenizing...\n");
    std::vector<uint32_t> tokens(text.size() + 1);
    size_t n = 0;
    const int ts = czg_tok_encode(L.tok, reinterpret_cast<const char *>(text.data()), text.size(), tokens.data(),
                                  tokens.size(), &n);
    if (ts == CZG_TOK_E_UTF8) die("stream did not contain valid UTF-8");
    if (ts != CZG_TOK_OK) die("tokenizer: status " + std::to_string(ts));
    tokens.resize(n);
    printf("  %zu bytes -> %zu tokens\n", text.size(), n);
    printf("Compressing...\n");
    const double te = now();
    int chunk = L.context_length;
    if (level > 0) {   // main.rs:113-122, 186-197
        const int req = level == 1 ? 64 : level == 2 ? 128 : level == 3 ? 256 : level == 4 ? 512 : 1024;
        if (req > L.context_length)
            fprintf(stderr, "Warning: Level %d requires %d tokens but model only supports %d. Using model's context length.\n",
                    level, req, L.context_length);
        else
            chunk = req;
    }
    uint32_t log2 = 0;
    while ((1 << (log2 + 1)) <= chunk) log2++;
    const size_t n_chunks = (n + (size_t)chunk - 1) / (size_t)chunk;
    std::vector<uint64_t> starts(n_chunks + 1);
    for (size_t i = 0; i <= n_chunks; i++) starts[i] = std::min<uint64_t>((uint64_t)i * (uint64_t)chunk, n);
    Container c;
    c.codec = codec;
    c.uncompressed_len = (uint32_t)text.size();
    c.model_id_hash = hash_model_path(model);
    c.log2 = log2 & 0xFF;
    c.last_chunk_tokens = (1u << c.log2) & 0xFFFF;
    if (n_chunks) {
        const uint64_t cap = czg_compress_bound(n, n_chunks);
        Bytes packed(cap);
        std::vector<uint32_t> lens(n_chunks);
        uint64_t used = 0;
        if (czg_compress_chunks(L.ctx, tokens.data(), starts.data(), (uint32_t)n_chunks, packed.data(), cap,
                                lens.data(), &used) != 0)
            die(std::string("engine: ") + czg_last_error(L.ctx));
        for (size_t i = 0; i < n_chunks; i++) {
            if (lens[i] > 0xFFFF) die("Chunk too large");   // file_format.rs:311
            c.lens.push_back(lens[i]);
        }
        c.last_chunk_tokens = (uint32_t)(starts[n_chunks] - starts[n_chunks - 1]) & 0xFFFF;
        c.data.assign(packed.begin(), packed.begin() + (ptrdiff_t)used);
    }
    const double t_enc = now() - te;
    printf("Writing output to '%s'...\n", out.c_str());
    Bytes outer;
    c.outer(outer);
    const Bytes body = outer_compress(c.payload(), codec);
    write_file(out, outer.data(), outer.size(), body.data(), body.size());
    const size_t ob = outer.size() + body.size();
    printf("\n=== Compression Results ===\n");
    printf("Input:  %zu bytes (%zu tokens)\n", text.size(), n);
    printf("Output: %zu bytes\n", ob);
    if (ob) printf("Ratio:  %.2fx (%.2f%%)\n", (double)text.size() / ob, 100.0 * ob / std::max<size_t>(1, text.size()));
    if (n) printf("Bits per token: %.2f\n", 8.0 * ob / n);
    printf("\nEncode time: %.2fs (%.1f tokens/sec)\n", t_enc, n / std::max(t_enc, 1e-9));
    printf("Total time:  %.2fs\n", now() - t0);
    return 0;
}

int do_decompress(const std::string &model, const std::string &tokp, const std::string &in, const std::string &out) {
    const double t0 = now();
    Loaded L;
    load(L, model, tokp, 0);
    printf("Reading compressed file from '%s'...\n", in.c_str());
    const Bytes file = read_file(in);
    Bytes payload;
    const Container c = Container::parse(file, payload);
    const size_t n_chunks = c.lens.size();
    std::vector<uint32_t> counts(n_chunks);
    std::vector<uint64_t> starts(n_chunks + 1, 0);
    uint64_t total = 0;
    for (size_t i = 0; i < n_chunks; i++) {
        counts[i] = c.chunk_tokens(i);
        total += counts[i];
        starts[i + 1] = starts[i] + c.lens[i];
    }
    printf("  %zu chunks, %llu tokens total\n", n_chunks, (unsigned long long)total);
    printf("Decompressing...\n");
    const double td = now();
    std::vector<uint32_t> tokens(total);
    if (n_chunks && czg_decompress_chunks(L.ctx, c.data.data(), starts.data(), counts.data(), (uint32_t)n_chunks,
                                          tokens.data()) != 0)
        die(std::string("engine: ") + czg_last_error(L.ctx));
    const double t_dec = now() - td;
    printf("Detokenizing...\n");
    size_t nb = 0;
    if (czg_tok_decode(L.tok, tokens.data(), tokens.size(), nullptr, 0, &nb) != CZG_TOK_OK)
        die(czg_tok_last_error(L.tok));
    Bytes bytes(nb + 1);
    if (czg_tok_decode(L.tok, tokens.data(), tokens.size(), bytes.data(), bytes.size(), &nb) != CZG_TOK_OK)
        die(czg_tok_last_error(L.tok));
    const std::string text = utf8_lossy(bytes.data(), nb);   // main.rs:405-412
    printf("Writing output to '%s'...\n", out.c_str());
    write_file(out, reinterpret_cast<const uint8_t *>(text.data()), text.size());
    printf("\n=== Decompression Results ===\n");
    printf("Tokens: %zu\n", tokens.size());
    printf("Output: %zu bytes\n", nb);
    printf("\nDecode time: %.2fs (%.1f tokens/sec)\n", t_dec, tokens.size() / std::max(t_dec, 1e-9));
    printf("Total time:  %.2fs\n", now() - t0);
    return 0;
}

// host parts without a GPU: MD5 vectors (RFC 1321 A.5), container and codec round trips, lossy UTF-8
int selftest() {
    const Md5 md5;
    const char *cases[][2] = {{"", "d41d8cd98f00b204e9800998ecf8427e"},
                              {"abc", "900150983cd24fb0d6963f7d28e17f72"},
                              {"message digest", "f96b697d7cb7938d525a2f31aaf161d0"},
                              {"12345678901234567890123456789012345678901234567890123456789012345678901234567890",
                               "57edf4a22be3c955ac49da2e2107b67a"}};
    for (auto &cs : cases)
        if (md5.hex(reinterpret_cast<const uint8_t *>(cs[0]), strlen(cs[0])) != cs[1]) die(std::string("md5 ") + cs[0]);
    Bytes sample;
    for (int i = 0; i < 70000; i++) sample.push_back((uint8_t)((i * 2654435761u) >> 27));
    for (int codec : {kZstd, kBrotli}) {
        Container c;
        c.codec = codec;
        c.uncompressed_len = 12345;
        c.model_id_hash = 0xDEADBEEF;
        c.log2 = 10;
        c.last_chunk_tokens = 77;
        for (int i = 0; i < 5; i++) {
            c.lens.push_back(1000 + i);
            c.data.insert(c.data.end(), sample.begin() + i * 1000, sample.begin() + i * 1000 + 1000 + i);
        }
        Bytes outer, payload;
        c.outer(outer);
        const Bytes body = outer_compress(c.payload(), codec);
        outer.insert(outer.end(), body.begin(), body.end());
        const Container d = Container::parse(outer, payload);
        if (d.codec != codec || d.lens != c.lens || d.data != c.data || d.last_chunk_tokens != 77 ||
            d.model_id_hash != 0xDEADBEEF || d.log2 != 10 || payload != c.payload())
            die("container round trip");
    }
    const uint8_t bad[] = {'a', 0xE2, 0x82, 'b', 0xF0, 0x9F, 0x98, 0x80, 0xC0, 0xAF, 0xED, 0xA0, 0x80};
    if (utf8_lossy(bad, sizeof(bad)) != "a\xEF\xBF\xBD" "b\xF0\x9F\x98\x80\xEF\xBF\xBD\xEF\xBF\xBD\xEF\xBF\xBD\xEF\xBF\xBD\xEF\xBF\xBD")
        die("utf8 lossy");
    printf("selftest ok: md5(\"%s\") prefix %08x\n", "models/v001_eng.czm", hash_model_path("models/v001_eng.czm"));
    return 0;
}

void usage() {
    fprintf(stderr,
            "usage: czg-cli compress   -m MODEL -i INPUT -o OUTPUT [-t TOKENIZER] [-c brotli|zstd] [-L 1..5]\n"
            "       czg-cli decompress -m MODEL -i INPUT -o OUTPUT [-t TOKENIZER]\n"
            "       czg-cli selftest\n"
            "       czg-cli outer zstd|brotli compress|decompress IN OUT\n"
            "       czg-cli md5-path PATH\n");
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 2) { usage(); return 2; }
    const std::string cmd = argv[1];
    try {
        if (cmd == "outer" && argc == 6) {
            const std::string c = argv[2], op = argv[3];
            const int codec = c == "zstd" ? kZstd : c == "brotli" ? kBrotli : -1;
            if (codec < 0 || (op != "compress" && op != "decompress")) { usage(); return 2; }
            const Bytes in = read_file(argv[4]);
            const Bytes o = op == "compress" ? outer_compress(in, codec) : outer_decompress(in, 0, codec);
            write_file(argv[5], o.data(), o.size());
            return 0;
        }
        if (cmd == "md5-path" && argc == 3) {
            printf("%08x\n", hash_model_path(argv[2]));
            return 0;
        }
    } catch (const std::exception &e) {
        fprintf(stderr, "Error: %s\n", e.what());
        return 1;
    }
    std::string model, tokp, in, out, codec = "brotli";
    int level = 0;
    for (int i = 2; i < argc; i++) {
        const std::string a = argv[i];
        auto val = [&](void) -> std::string {
            if (i + 1 >= argc) { usage(); exit(2); }
            return argv[++i];
        };
        if (a == "-m" || a == "--model") model = val();
        else if (a == "-t" || a == "--tokenizer") tokp = val();
        else if (a == "-i" || a == "--input") in = val();
        else if (a == "-o" || a == "--output") out = val();
        else if ((a == "-c" || a == "--codec") && cmd == "compress") codec = val();
        else if ((a == "-L" || a == "--level") && cmd == "compress") {
            level = atoi(val().c_str());
            if (level < 1 || level > 5) { usage(); return 2; }
        } else { usage(); return 2; }
    }
    try {
        if (cmd == "selftest") return selftest();
        if (model.empty() || in.empty() || out.empty()) { usage(); return 2; }
        for (auto &ch : codec) ch = (char)tolower(ch);
        if (cmd == "compress") return do_compress(model, tokp, in, out, codec, level);
        if (cmd == "decompress") return do_decompress(model, tokp, in, out);
        usage();
        return 2;
    } catch (const std::exception &e) {   // main.rs:450-453: print the error, exit 1
        fprintf(stderr, "Error: %s\n", e.what());
        return 1;
    }
}
