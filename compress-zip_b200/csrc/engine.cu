// engine.cu -- the C-ABI context: model upload, wave scheduling of chunk
// batches through the sm_100a kernels, statistics.  Declared in include/czg.h.
//
// A compress call (the chunk loop of rust/src/main.rs:206-238 for all chunks at
// once) runs in waves of consecutive chunks.  Rows of a wave are the wave's
// tokens in input order, so chunk c of the wave owns rows
// [starts[c] - starts[c0], starts[c+1] - starts[c0]).  Per wave:
//   rows -> embed+norm1 -> per layer {QKV GEMM+requant -> K RoPE/V stage ->
//   exact attention -> O GEMM+requant -> norm3+residual+norm2 -> up GEMM+requant
//   +ReGLU -> down GEMM+requant -> norm4+residual+next norm} -> LM head GEMM
//   (int32 logits) -> CDF reduced to the coder interval -> one encoder thread per
//   chunk -> pack.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "czg.h"
#include "czm_parse.h"
#include "kernels.h"

using namespace czg;

void czg::kernels_init() {
    attention_init();
    attention_mma_init();
    gemm_tc_init();
    gemm_norm_init();
    head_cdf_init();
}

namespace {

enum KernelClass {
    kRows = 0, kEmbedNorm, kGemmQkv, kKvPrep, kAttention, kGemmO, kResidualNorm, kGemmUp,
    kGemmDown, kGemmHead, kCdf, kEncode, kPack, kKvAppend, kAttnDecode, kCdfDecode, kHeadCdf,
    kGemmONorm, kGemmDownNorm, kNumClasses
};
static_assert(kNumClasses <= CZG_MAX_KERNEL_CLASSES, "too many kernel classes");
const char *kClassNames[kNumClasses] = {
    "rows", "embed_norm", "gemm_qkv", "kv_prep", "attention", "gemm_o", "residual_norm",
    "gemm_up_reglu", "gemm_down", "gemm_head", "cdf", "encode", "pack", "kv_append",
    "attention_decode", "cdf_decode", "head_cdf", "gemm_o_norm", "gemm_down_norm"};

thread_local std::string g_create_error;

struct LayerDev {
    int8_t *attn_norm = nullptr, *post_attn_norm = nullptr, *ffn_norm = nullptr,
           *post_ffn_norm = nullptr;
    int8_t *qkv_w = nullptr, *out_w = nullptr, *up_w = nullptr, *down_w = nullptr;
    int32_t *score_mult = nullptr;
    int8_t *sink_key = nullptr;
    // attention score arithmetic: 0 exact FP32 (every |score_mult| < 2^19), 1 32-bit
    // integer (< 2^27), 2 64-bit with saturation (any)
    int score_mode = 0;
    int qkv_mult = 1, out_mult = 1, up_mult = 1, down_mult = 1;
    int qkv_shift = 0, out_shift = 0, up_shift = 0, down_shift = 0;
    TcMatrix tm_qkv, tm_out, tm_up, tm_down;   // TMA descriptors of the weights
    // O / down projection with the residual norm in the epilogue (gemm_norm.cu): the
    // weights read in boxes of d/2 rows; chosen at model load when the projection has
    // the FP32 requantisation form and d is 256, 384 or 512 (else the GEMM and
    // k_residual_norm run apart)
    TcMatrix tm_out_h, tm_down_h;
    bool fused_o = false, fused_down = false;
};

struct EvPair {
    cudaEvent_t a, b;
    int cls;
};

}  // namespace

struct czg_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;       // stream all work runs on
    cudaStream_t own_stream = nullptr;   // the context's own stream
    std::string err;
    czg_model_info info{};
    int eps = 1;
    bool scalar_attention = false;   // CZG_SCALAR_ATTENTION=1 selects the CUDA-core kernel
    bool staged_attention = false;   // CZG_ATTN_STAGED=1: chunks <= 1024 keys with K/V^T staged in shared memory
    int vpad = 0;           // vocab rounded up to the GEMM tile (extra head rows are zero)
    int dff_pad = 0;        // d_ff rounded up to the GEMM tile (extra hidden units are zero)
    int8_t *embed = nullptr, *final_norm = nullptr, *head_w = nullptr;
    int8_t *xn_tab = nullptr;   // [V][d]: the first pre-norm of every token's embedding row
    uint16_t *lut = nullptr;
    uint16_t *lut4k = nullptr;   // exp_q16 by t256 <= 4096 (lut.rs:213-235 unrolled over ip)
    uint16_t *inv_tab = nullptr;   // inv_rms_q15 by floor(sum_sq / d), eps folded in
    bool kernel_timing = false;   // CUDA events around every kernel (czg_set_kernel_timing, CZG_KERNEL_TIMING=1)
    bool exp0 = false;           // lut4k[0] == 65535: exp of a zero difference needs no special case
    bool logit_small = false;    // every |logit| < 2^30: no logit difference wraps
    bool head_cdf = false;       // the fused head GEMM + coder interval kernel applies
    bool gemm_failed = false;    // a GEMM launch was refused (shape or output map); the call fails
    int16_t *rope_cos = nullptr, *rope_sin = nullptr;
    std::vector<LayerDev> layers;
    std::vector<void *> allocs;

    // wave workspace (grown on demand up to wave_cap rows)
    int cap_rows = 0, cap_chunks = 0, wave_cap = 0;
    std::vector<void *> ws_allocs;
    uint32_t *tokens = nullptr, *tok_in = nullptr, *tok_out = nullptr;
    int *pos = nullptr, *x_res = nullptr, *err_flag = nullptr;
    int *task_ctr = nullptr;   // the streamed attention's global task counter
    bool res16 = false;   // residual stream stored as int16 (exact for n_layers <= 128)
    int8_t *xn = nullptr, *qkv = nullptr, *kv = nullptr, *attn = nullptr, *o8 = nullptr, *hbuf = nullptr;
    int32_t *logits = nullptr;
    uint2 *lohi = nullptr;
    uint8_t *slots = nullptr, *packed = nullptr;
    uint32_t *lens = nullptr;
    uint64_t *slot_off = nullptr, *pack_off = nullptr, *chunk_tok0 = nullptr;
    int *chunk_row0 = nullptr, *chunk_len = nullptr;
    int *att_row0 = nullptr, *att_len = nullptr;   // the chunks in attention launch order
    int *att_kvoff = nullptr;                        // and their streaming K/V offsets (128-byte units)
    int *rowchunk = nullptr;                         // chunk of each row of a wave
    // TMA descriptors of the GEMM A operands (wave buffers) and the head
    TcMatrix tm_xn, tm_attn, tm_h, tm_head;
    // decompression buffers (grown on demand)
    size_t dec_streams = 0, dec_len = 0, dec_bytes = 0, dec_tokens = 0;
    int8_t *kvc = nullptr;
    DecState *dstate = nullptr;
    uint8_t *ddata = nullptr;
    uint64_t *d_off = nullptr, *d_len = nullptr, *d_tokoff = nullptr;
    uint32_t *d_outtok = nullptr;
    std::vector<void *> dec_allocs;
    // pinned staging of the decoded tokens (grown on demand)
    uint8_t *h_out = nullptr;
    size_t h_out_bytes = 0;
    // pinned host staging: chunk tables of the wave being launched (two, so a wave's
    // tables can be written while the previous wave's copies are still queued), and
    // per wave parity the error word, packed total and chunk lengths copied back
    uint8_t *h_meta = nullptr, *h_meta2 = nullptr, *h_meta_cur = nullptr;
    uint8_t *h_small[2] = {nullptr, nullptr};
    std::vector<int> att_order;
    size_t h_meta_bytes = 0;
    // copy-out pipeline of compress calls: a second token buffer and packed buffer,
    // a stream for the copies and the events that order them with the compute stream
    uint32_t *tokens2 = nullptr;
    uint8_t *packed2 = nullptr;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_h2d[2] = {nullptr, nullptr}, ev_comp[2] = {nullptr, nullptr};
    cudaEvent_t ev_small[2] = {nullptr, nullptr}, ev_d2h[2] = {nullptr, nullptr};

    // statistics
    czg_stats stats{};
    std::vector<EvPair> evs;
    size_t ev_used = 0;
    cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
};

namespace {

int fail(czg_ctx *c, int code, const std::string &msg) {
    if (c) c->err = msg;
    else g_create_error = msg;
    return code;
}

bool cuda_ok(czg_ctx *c, cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    c->err = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
}

template <class T>
bool dalloc(czg_ctx *c, T **p, size_t n) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(n, 16) * sizeof(T));
    if (e != cudaSuccess) {
        c->err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
        return false;
    }
    c->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return true;
}

template <class T>
bool dalloc_ws(czg_ctx *c, T **p, size_t n) {
    if (!dalloc(c, p, n)) return false;
    c->ws_allocs.push_back(c->allocs.back());   // freed with the workspace
    c->allocs.pop_back();
    return true;
}

template <class T>
bool upload(czg_ctx *c, T **p, const void *src, size_t bytes) {
    if (!dalloc(c, reinterpret_cast<uint8_t **>(p), bytes)) return false;
    return cuda_ok(c, cudaMemcpy(*p, src, bytes, cudaMemcpyHostToDevice), "upload");
}

EvPair &next_ev(czg_ctx *c, int cls) {
    if (c->ev_used == c->evs.size()) {
        EvPair e;
        cudaEventCreate(&e.a);
        cudaEventCreate(&e.b);
        c->evs.push_back(e);
    }
    EvPair &e = c->evs[c->ev_used++];
    e.cls = cls;
    return e;
}

struct PdlScope {   // g_pdl_launch on for the scope's lifetime
    explicit PdlScope(bool on) { g_pdl_launch = on; }
    ~PdlScope() { g_pdl_launch = false; }
    PdlScope(const PdlScope &) = delete;
    PdlScope &operator=(const PdlScope &) = delete;
};

template <class F>
void timed(czg_ctx *c, int cls, F &&f) {
    c->stats.launches[cls]++;
    if (!c->kernel_timing) {
        f();
        return;
    }
    EvPair &e = next_ev(c, cls);
    cudaEventRecord(e.a, c->stream);
    f();
    cudaEventRecord(e.b, c->stream);
}

// Accumulate the recorded event pairs (class -1 = H2D copy, -2 = D2H copy).
void collect_events(czg_ctx *c) {
    for (size_t i = 0; i < c->ev_used; i++) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, c->evs[i].a, c->evs[i].b) != cudaSuccess) continue;
        int cls = c->evs[i].cls;
        if (cls == -1) c->stats.h2d_ms += ms;
        else if (cls == -2) c->stats.d2h_ms += ms;
        else c->stats.kernel_ms[cls] += ms;
    }
    c->ev_used = 0;
}

// ---- model loading --------------------------------------------------------

int meta_int(const CzmFile &f, const char *key, int dflt) {
    auto it = f.metadata.find(key);
    if (it == f.metadata.end()) return dflt;
    const std::string &s = it->second;
    if (s.empty()) return dflt;
    char *endp = nullptr;
    long long v = strtoll(s.c_str(), &endp, 10);
    if (*endp != '\0' || v < 0 || v > 0x7fffffff) return dflt;   // usize parse failure
    return (int)v;
}

const TensorRef *find(const CzmFile &f, const std::string &name) {
    auto it = f.tensors.find(name);
    return it == f.tensors.end() ? nullptr : &it->second;
}

int need(czg_ctx *c, const CzmFile &f, const std::string &name, const char *dtype, int64_t numel,
         const TensorRef **out) {
    const TensorRef *t = find(f, name);
    if (!t) return fail(c, CZG_E_MODEL, "Missing tensor: " + name);
    if (t->dtype != dtype) return fail(c, CZG_E_MODEL, "tensor " + name + " has dtype " + t->dtype +
                                              ", expected " + dtype);
    size_t esz = t->dtype == "I8" || t->dtype == "U8" ? 1 : (t->dtype == "I16" || t->dtype == "U16" ? 2 : 4);
    if (t->numel() < numel || (size_t)t->numel() * esz > t->nbytes)
        return fail(c, CZG_E_MODEL, "tensor " + name + " is too small");
    *out = t;
    return CZG_OK;
}

// model.rs:157-170: a missing *.mult reads as 1, a missing *.shift as 0
int scalar_i32(czg_ctx *c, const CzmFile &f, const std::string &name, int dflt, int *out) {
    const TensorRef *t = find(f, name);
    if (!t) { *out = dflt; return CZG_OK; }
    if (t->dtype != "I32" || t->nbytes < 4) return fail(c, CZG_E_MODEL, "tensor " + name + " is not I32");
    int32_t v;
    memcpy(&v, t->data, 4);
    *out = v;
    return CZG_OK;
}

int scalar_i8(czg_ctx *c, const CzmFile &f, const std::string &name, int dflt, int *out) {
    const TensorRef *t = find(f, name);
    if (!t) { *out = dflt; return CZG_OK; }
    if (t->dtype != "I8" || t->nbytes < 1) return fail(c, CZG_E_MODEL, "tensor " + name + " is not I8");
    *out = (int8_t)t->data[0];
    return CZG_OK;
}

int load_model(czg_ctx *c, const uint8_t *bytes, size_t len) {
    CzmFile f;
    std::string perr = parse_czm(bytes, len, f);
    if (!perr.empty()) return fail(c, CZG_E_MODEL, "Failed to load safetensors: " + perr);
    czg_model_info &m = c->info;
    // model.rs:113-145
    int ctx = meta_int(f, "context_length", -1);
    if (ctx < 0) {
        int l2 = meta_int(f, "context_length_log2", -1);
        ctx = l2 >= 0 && l2 < 31 ? (1 << l2) : meta_int(f, "max_seq_len", 64);
    }
    m.vocab_size = meta_int(f, "vocab_size", 1024);
    m.n_layers = meta_int(f, "n_layers", 1);
    m.n_heads = meta_int(f, "n_heads", 6);
    m.n_kv_heads = meta_int(f, "n_kv_heads", 1);
    m.d_model = meta_int(f, "d_model", 384);
    m.d_ff = meta_int(f, "d_ff", 1024);
    m.head_dim = meta_int(f, "head_dim", 64);
    m.max_seq_len = meta_int(f, "max_seq_len", 64);
    m.context_length = ctx;
    const int d = m.d_model, V = m.vocab_size, H = m.n_heads, dff = m.d_ff;
    // shapes the reference runs without panicking (attention.rs:172-176, main.rs:214)
    if (!(H == 4 || H == 6 || H == 8)) return fail(c, CZG_E_UNSUPPORTED, "n_heads must be 4, 6 or 8");
    if (m.head_dim != 64 || d != H * 64) return fail(c, CZG_E_UNSUPPORTED, "head_dim must be 64 and d_model = 64 * n_heads");
    if (m.n_kv_heads < 1 || (d + 2 * 64 * m.n_kv_heads) / (d + 128) != 1)
        return fail(c, CZG_E_UNSUPPORTED, "n_kv_heads gives a KV batch other than 1");
    if (V <= 1022 || V > 65536) return fail(c, CZG_E_UNSUPPORTED, "vocab_size must be in 1023..65536");
    if (m.n_layers < 1 || m.n_layers > 256) return fail(c, CZG_E_UNSUPPORTED, "n_layers out of range");
    if (dff < 64 || dff % 64 != 0 || dff > 16384) return fail(c, CZG_E_UNSUPPORTED, "d_ff must be a multiple of 64");
    if (ctx < 1 || ctx > 65536) return fail(c, CZG_E_UNSUPPORTED, "context_length out of range");
    const int qkv_rows = d + 2 * 64 * m.n_kv_heads;
    int st;
    const TensorRef *t;
    if ((st = need(c, f, "embed.weight", "I8", (int64_t)V * d, &t))) return st;
    if (!upload(c, &c->embed, t->data, (size_t)V * d)) return CZG_E_DEVICE;
    if ((st = need(c, f, "norm.weight", "I8", d, &t))) return st;
    if (!upload(c, &c->final_norm, t->data, d)) return CZG_E_DEVICE;
    if ((st = need(c, f, "head.weight", "I8", (int64_t)V * d, &t))) return st;
    c->vpad = (V + 127) / 128 * 128;
    {
        std::vector<int8_t> hp((size_t)c->vpad * d, 0);
        memcpy(hp.data(), t->data, (size_t)V * d);
        if (!upload(c, &c->head_w, hp.data(), hp.size())) return CZG_E_DEVICE;
    }
    if ((st = need(c, f, "lut.exp2", "U16", 256, &t))) return st;
    if (t->numel() != 256) return fail(c, CZG_E_MODEL, "Exp2 LUT must have exactly 256 entries");
    if (!upload(c, &c->lut, t->data, 512)) return CZG_E_DEVICE;
    {   // t256 -> clamp(((65536 >> (t256 >> 8)) * lut[t256 & 255] + 2^15) >> 16, 1, 65535)
        uint16_t lut8[256];
        memcpy(lut8, t->data, 512);
        std::vector<uint16_t> l4(4104, 1);   // entries 4096.. are 1: every t256 >= 4096 gives 1
        for (uint32_t tt = 0; tt < 4096; tt++) {
            uint32_t o = (((1u << 16) >> (tt >> 8)) * (uint32_t)lut8[tt & 255] + 0x8000u) >> 16;
            l4[tt] = (uint16_t)std::min(65535u, std::max(1u, o));
        }
        if (!upload(c, &c->lut4k, l4.data(), l4.size() * 2)) return CZG_E_DEVICE;
        c->exp0 = l4[0] == 65535;
    }
    if (!dalloc(c, &c->inv_tab, (size_t)kInvTabEntries)) return CZG_E_DEVICE;
    launch_inv_table(c->eps, c->inv_tab, c->stream);
    for (int k = 0; k < 2; k++) {
        const char *nm = k ? "lut.rope_sin" : "lut.rope_cos";
        if ((st = need(c, f, nm, "I16", (int64_t)ctx * 32, &t))) return st;
        if (t->numel() != (int64_t)ctx * 32)   // model.rs:325-333 (from_arrays_with_dims)
            return fail(c, CZG_E_MODEL, "RoPE LUT arrays size mismatch with max_seq_len * half_dim");
        if (!upload(c, k ? &c->rope_sin : &c->rope_cos, t->data, (size_t)ctx * 64)) return CZG_E_DEVICE;
    }
    // softmax constants (model.rs:255-262, fallbacks softmax_cdf.rs:23-46)
    const TensorRef *tc = find(f, "softmax.coef_q24"), *tt = find(f, "softmax.target_total");
    if (tc && (tc->dtype != "U32" || tc->nbytes < 4)) return fail(c, CZG_E_MODEL, "softmax.coef_q24 is not U32");
    if (tt && (tt->dtype != "U32" || tt->nbytes < 4)) return fail(c, CZG_E_MODEL, "softmax.target_total is not U32");
    if (tc) memcpy(&m.coef_q24, tc->data, 4);
    else m.coef_q24 = (uint32_t)std::max(1.0, std::round((0.1 * 1.4426950408889634) / 64.0 * 16777216.0));
    if (tt) memcpy(&m.target_total, tt->data, 4);
    else {
        uint32_t q = 1u << 30, vs = (uint32_t)V;
        uint32_t tgt = q > vs ? q - vs : 0;
        tgt = tgt > 1024 ? tgt - 1024 : 0;
        m.target_total = std::max(tgt, vs + 1);
    }
    if (m.target_total <= (uint32_t)V || m.target_total >= (1u << 30))
        return fail(c, CZG_E_UNSUPPORTED, "softmax.target_total must lie in (vocab_size, 2^30)");

    // The tcgen05 GEMMs take K and N in multiples of 128.  d = 64 * n_heads is one
    // (n_heads 4, 6, 8 give 256, 384, 512); d_ff (a multiple of 64) is padded to dffp
    // with zero gate/up rows and zero down columns: requant(0) = 0 and ReGLU(0, 0) = 0,
    // so the padded hidden units are 0 and add nothing to the down projection.
    const int dffp = (dff + 127) / 128 * 128;
    c->dff_pad = dffp;
    c->layers.resize(m.n_layers);
    c->logit_small = (long long)d * 127 * 128 < (1ll << 30);   // |logit| <= d * 127 * 128
    c->res16 = m.n_layers <= 128 && getenv("CZG_RESIDUAL32") == nullptr;
    for (int i = 0; i < m.n_layers; i++) {
        LayerDev &L = c->layers[i];
        std::string p = "layers." + std::to_string(i) + ".";
        struct { const char *nm; int8_t **dst; } norms[4] = {
            {"attn_norm.weight", &L.attn_norm}, {"post_attn_norm.weight", &L.post_attn_norm},
            {"ffn_norm.weight", &L.ffn_norm}, {"post_ffn_norm.weight", &L.post_ffn_norm}};
        for (auto &nw : norms) {
            if ((st = need(c, f, p + nw.nm, "I8", d, &t))) return st;
            if (!upload(c, nw.dst, t->data, d)) return CZG_E_DEVICE;
        }
        if ((st = need(c, f, p + "attn.qkv.weight", "I8", (int64_t)qkv_rows * d, &t))) return st;
        // only rows [0, d + 128) are read: q, then the single K and V the reference uses
        if (!upload(c, &L.qkv_w, t->data, (size_t)(d + 128) * d)) return CZG_E_DEVICE;
        if ((st = need(c, f, p + "attn.out.weight", "I8", (int64_t)d * d, &t))) return st;
        if (!upload(c, &L.out_w, t->data, (size_t)d * d)) return CZG_E_DEVICE;
        if ((st = need(c, f, p + "ffn.up.weight", "I8", (int64_t)2 * dff * d, &t))) return st;
        {   // interleave gate row j and up row j so the GEMM epilogue sees both; rows
            // j >= d_ff (padding to dffp) stay zero
            std::vector<int8_t> il((size_t)2 * dffp * d, 0);
            for (int j = 0; j < dff; j++) {
                memcpy(&il[(size_t)(2 * j) * d], t->data + (size_t)j * d, d);
                memcpy(&il[(size_t)(2 * j + 1) * d], t->data + (size_t)(dff + j) * d, d);
            }
            if (!upload(c, &L.up_w, il.data(), il.size())) return CZG_E_DEVICE;
        }
        if ((st = need(c, f, p + "ffn.down.weight", "I8", (int64_t)d * dff, &t))) return st;
        {   // [d][dffp]: columns j >= d_ff are zero
            std::vector<int8_t> dw((size_t)d * dffp, 0);
            for (int i = 0; i < d; i++) memcpy(&dw[(size_t)i * dffp], t->data + (size_t)i * dff, dff);
            if (!upload(c, &L.down_w, dw.data(), dw.size())) return CZG_E_DEVICE;
        }
        if ((st = need(c, f, p + "attn.score_mult", "I32", H, &t))) return st;
        if (!upload(c, &L.score_mult, t->data, (size_t)H * 4)) return CZG_E_DEVICE;
        for (int hh = 0; hh < H; hh++) {
            int32_t sm;
            memcpy(&sm, t->data + 4 * hh, 4);
            const long long am = sm < 0 ? -(long long)sm : (long long)sm;
            L.score_mode = std::max(L.score_mode, am >= (1ll << 27) ? 2 : (am >= (1ll << 19) ? 1 : 0));
        }
        if (const TensorRef *sk = find(f, p + "attn.sink_key")) {
            if (sk->dtype != "I8" || sk->numel() < 64 || sk->nbytes < 64)
                return fail(c, CZG_E_MODEL, "attn.sink_key must be I8[64]");
            if (!upload(c, &L.sink_key, sk->data, 64)) return CZG_E_DEVICE;
        }
        if ((st = scalar_i32(c, f, p + "attn.qkv.mult", 1, &L.qkv_mult))) return st;
        if ((st = scalar_i32(c, f, p + "attn.out.mult", 1, &L.out_mult))) return st;
        if ((st = scalar_i32(c, f, p + "ffn.up.mult", 1, &L.up_mult))) return st;
        if ((st = scalar_i32(c, f, p + "ffn.down.mult", 1, &L.down_mult))) return st;
        if ((st = scalar_i8(c, f, p + "attn.qkv.shift", 0, &L.qkv_shift))) return st;
        if ((st = scalar_i8(c, f, p + "attn.out.shift", 0, &L.out_shift))) return st;
        if ((st = scalar_i8(c, f, p + "ffn.up.shift", 0, &L.up_shift))) return st;
        if ((st = scalar_i8(c, f, p + "ffn.down.shift", 0, &L.down_shift))) return st;
        const char *fn = getenv("CZG_FUSED_NORM");
        const bool fuse = gemm_norm_supported(d) && !(fn && std::string(fn) == "0");
        float mf, c2;
        int ca;
        // (the fused kernels use the FP32 requantisation, which needs |acc| < 2^29)
        L.fused_o = fuse && (long long)d * 16256 < (1ll << 29) && requant_fp32(L.out_mult, L.out_shift, &mf, &c2, &ca);
        L.fused_down = fuse && (long long)dffp * 16256 < (1ll << 29) &&
                       requant_fp32(L.down_mult, L.down_shift, &mf, &c2, &ca);
    }
    {   // the first pre-norm depends on the token alone: one row per vocabulary entry
        std::vector<uint32_t> iota(V);
        for (int v = 0; v < V; v++) iota[v] = (uint32_t)v;
        uint32_t *d_iota = nullptr;
        if (!upload(c, &d_iota, iota.data(), (size_t)V * 4) || !dalloc(c, &c->xn_tab, (size_t)V * d))
            return CZG_E_DEVICE;
        launch_embed_norm(d_iota, c->embed, c->layers[0].attn_norm, V, d, c->inv_tab, nullptr, c->res16, false,
                          c->xn_tab, c->stream);
        if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "normalised embedding table")) return CZG_E_DEVICE;
    }
    return CZG_OK;
}

// device bytes of the wave workspace per row (the per-chunk arrays are small)
size_t workspace_row_bytes(const czg_ctx *c) {
    const czg_model_info &m = c->info;
    const size_t d = (size_t)m.d_model;
    return 16 + 4 * d + d + (d + 128) + 128 + d + d + (size_t)c->dff_pad + 4 * (size_t)c->vpad + 8 + 4 + 4;
}

// (Re)allocate the wave workspace for `rows` tokens and `chunks` chunks per wave;
// the previous workspace, if any, is released after the stream drains.
int alloc_workspace(czg_ctx *c, int rows, int chunks) {
    const czg_model_info &m = c->info;
    const int d = m.d_model;
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (void *p : c->ws_allocs) cudaFree(p);
    c->ws_allocs.clear();
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    for (uint8_t **h : {&c->h_meta, &c->h_meta2, &c->h_small[0], &c->h_small[1]}) {
        if (*h) cudaFreeHost(*h);
        *h = nullptr;
    }
    c->cap_rows = c->cap_chunks = 0;
    size_t R = (size_t)(rows + 127) / 128 * 128 + 128;
    bool ok = dalloc_ws(c, &c->tokens, R) && dalloc_ws(c, &c->tok_in, R) && dalloc_ws(c, &c->tok_out, R) &&
              dalloc_ws(c, &c->pos, R) && dalloc_ws(c, &c->x_res, R * d) && dalloc_ws(c, &c->xn, R * d) &&
              dalloc_ws(c, &c->qkv, R * (d + 128)) && dalloc_ws(c, &c->kv, R * 128 + (size_t)chunks * 4096) &&
              dalloc_ws(c, &c->rowchunk, R) &&
              dalloc_ws(c, &c->attn, R * d) && dalloc_ws(c, &c->o8, R * d) &&
              dalloc_ws(c, &c->hbuf, R * c->dff_pad) && dalloc_ws(c, &c->logits, R * c->vpad) &&
              dalloc_ws(c, &c->lohi, R) && dalloc_ws(c, &c->slots, 4 * R + 8 * (size_t)chunks + 64) &&
              dalloc_ws(c, &c->packed, 4 * R + 8 * (size_t)chunks + 64) &&
              dalloc_ws(c, &c->packed2, 4 * R + 8 * (size_t)chunks + 64) && dalloc_ws(c, &c->tokens2, R) &&
              dalloc_ws(c, &c->lens, (size_t)chunks) && dalloc_ws(c, &c->slot_off, (size_t)chunks + 1) &&
              dalloc_ws(c, &c->pack_off, (size_t)chunks + 1) && dalloc_ws(c, &c->chunk_tok0, (size_t)chunks) &&
              dalloc_ws(c, &c->chunk_row0, (size_t)chunks) && dalloc_ws(c, &c->chunk_len, (size_t)chunks) &&
              dalloc_ws(c, &c->att_row0, (size_t)chunks) && dalloc_ws(c, &c->att_len, (size_t)chunks) &&
              dalloc_ws(c, &c->att_kvoff, (size_t)chunks) &&
              dalloc_ws(c, &c->err_flag, 1) && dalloc_ws(c, &c->task_ctr, 1);
    if (!ok) return CZG_E_DEVICE;
    cudaMemsetAsync(c->err_flag, 0, sizeof(int), c->stream);
    c->cap_rows = rows;
    c->cap_chunks = chunks;
    // TMA descriptors of every GEMM operand (d, d + 128, 2 * dff_pad and vpad are
    // multiples of 128 by construction)
    const int dffp = c->dff_pad;
    bool maps = tc_make_matrix(c->tm_xn, c->xn, R, d, 128) && tc_make_matrix(c->tm_attn, c->attn, R, d, 128) &&
                tc_make_matrix(c->tm_h, c->hbuf, R, dffp, 128) &&
                tc_make_matrix(c->tm_head, c->head_w, c->vpad, d, tc_bn_for(c->vpad));
    for (auto &L : c->layers) {
        maps = maps && tc_make_matrix(L.tm_qkv, L.qkv_w, d + 128, d, tc_bn_for(d + 128)) &&
               tc_make_matrix(L.tm_out, L.out_w, d, d, tc_bn_for(d)) &&
               tc_make_matrix(L.tm_out_h, L.out_w, d, d, d / 2) && tc_make_matrix(L.tm_down_h, L.down_w, d, dffp, d / 2) &&
               tc_make_matrix(L.tm_up, L.up_w, 2 * dffp, d, tc_bn_for(2 * dffp)) &&
               tc_make_matrix(L.tm_down, L.down_w, d, dffp, tc_bn_for(d));
    }
    if (!maps) return fail(c, CZG_E_DEVICE, "cuTensorMapEncodeTiled failed for a GEMM operand");
    // fused head + coder interval: the shipped exp table, |logit| < 2^30, V a multiple of 256
    const char *hc = getenv("CZG_HEAD_CDF");
    c->head_cdf = !(hc && std::string(hc) == "0") && c->exp0 && c->logit_small &&
                  m.vocab_size == c->vpad && c->vpad % 256 == 0 && m.coef_q24 < (1u << 23) && d % 128 == 0;
    c->h_meta_bytes = (size_t)chunks * 48 + 64;
    if (!cuda_ok(c, cudaMallocHost(&c->h_meta, c->h_meta_bytes), "cudaMallocHost") ||
        !cuda_ok(c, cudaMallocHost(&c->h_meta2, c->h_meta_bytes), "cudaMallocHost") ||
        !cuda_ok(c, cudaMallocHost(&c->h_small[0], 16 + 4 * (size_t)chunks), "cudaMallocHost") ||
        !cuda_ok(c, cudaMallocHost(&c->h_small[1], 16 + 4 * (size_t)chunks), "cudaMallocHost"))
        return CZG_E_DEVICE;
    c->h_meta_cur = c->h_meta;
    return CZG_OK;
}

// Grow the workspace to hold `rows` tokens per wave (at most wave_cap, and at most
// ~40% of the free device memory); small calls keep a small workspace.
int ensure_workspace(czg_ctx *c, size_t rows) {
    rows = std::min<size_t>(rows, (size_t)c->wave_cap);
    if (rows <= (size_t)c->cap_rows) return CZG_OK;
    size_t want = std::min<size_t>((size_t)c->wave_cap, std::max<size_t>(rows, 2 * (size_t)c->cap_rows));
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
        // the current workspace is released first, so it counts as free
        const size_t have = (size_t)c->cap_rows * workspace_row_bytes(c);
        const size_t fit = (size_t)((free_b + have) * 0.4) / workspace_row_bytes(c);
        want = std::max<size_t>((size_t)c->cap_rows, std::min(want, fit));
    }
    if (want <= (size_t)c->cap_rows) return CZG_OK;
    const int rows_i = (int)want;
    return alloc_workspace(c, rows_i, std::max(1024, rows_i / 16));
}

// One projection on the tcgen05 GEMM.  A shape it cannot take or an output map
// that cannot be encoded is an error of the call (there is no other GEMM).
bool gemm(czg_ctx *c, const TcMatrix &ta, const TcMatrix &tb, int M, int N, int K, int epi, int mult, int shift,
          void *out, int ldo, const KvSplit *kvs = nullptr) {
    if (launch_gemm_tc(ta, tb, M, N, K, epi, mult, shift, out, ldo, c->err_flag, c->stream, kvs)) return true;
    c->gemm_failed = true;
    return false;
}

// Attention output -> O projection -> post-attention norm, residual add (layer 0:
// from the embedding row) and the FFN pre-norm into xn (model.rs:418-438): one
// fused kernel, or the GEMM and k_residual_norm.
void o_norm(czg_ctx *c, const LayerDev &L, int l, int M, cudaStream_t st) {
    const int d = c->info.d_model;
    const int8_t *embed = l == 0 ? c->embed : nullptr;
    if (L.fused_o) {
        timed(c, kGemmONorm, [&] {
            if (!launch_gemm_norm(c->tm_attn, L.tm_out_h, M, d, d, L.out_mult, L.out_shift, L.ffn_norm,
                                  L.post_attn_norm, c->inv_tab, c->tok_in, embed, true, c->x_res, c->res16, c->xn,
                                  c->err_flag, st))
                c->gemm_failed = true;
        });
        return;
    }
    timed(c, kGemmO, [&] { gemm(c, c->tm_attn, L.tm_out, M, d, d, kEpiRequant, L.out_mult, L.out_shift, c->o8, d); });
    timed(c, kResidualNorm, [&] {
        launch_residual_norm(c->o8, L.ffn_norm, L.post_attn_norm, M, d, c->inv_tab, c->tok_in, embed, true,
                             c->x_res, c->res16, c->xn, st);
    });
}

// FFN hidden -> down projection -> post-FFN norm, residual add and the next layer's
// pre-norm (or the final norm; the residual is then not stored) (model.rs:455-475).
void down_norm(czg_ctx *c, const LayerDev &L, int l, int M, cudaStream_t st) {
    const czg_model_info &m = c->info;
    const int d = m.d_model;
    const int8_t *next = l + 1 < m.n_layers ? c->layers[l + 1].attn_norm : c->final_norm;
    const bool store = l + 1 < m.n_layers;
    if (L.fused_down) {
        timed(c, kGemmDownNorm, [&] {
            if (!launch_gemm_norm(c->tm_h, L.tm_down_h, M, d, c->dff_pad, L.down_mult, L.down_shift,
                                  L.post_ffn_norm, next, c->inv_tab, c->tok_in, nullptr, store, c->x_res, c->res16,
                                  c->xn, c->err_flag, st))
                c->gemm_failed = true;
        });
        return;
    }
    timed(c, kGemmDown, [&] {
        gemm(c, c->tm_h, L.tm_down, M, d, c->dff_pad, kEpiRequant, L.down_mult, L.down_shift, c->o8, d);
    });
    timed(c, kResidualNorm, [&] {
        launch_residual_norm(c->o8, L.post_ffn_norm, next, M, d, c->inv_tab, c->tok_in, nullptr, store, c->x_res,
                             c->res16, c->xn, st);
    });
}

struct Trace {
    int32_t *logits = nullptr;
    uint32_t *lohi = nullptr;
    int8_t *attn = nullptr;
    int8_t *final_in = nullptr;
};

// Chunk tables of the wave [c0, c1) to the device: row offset, length, token
// offset, slot offsets, and the chunks in attention launch order.  Returns the
// longest chunk.
int wave_meta(czg_ctx *c, const uint64_t *starts, uint32_t c0, uint32_t c1) {
    const int nc = (int)(c1 - c0);
    cudaStream_t st = c->stream;
    int *h_row0 = reinterpret_cast<int *>(c->h_meta_cur);
    int *h_len = h_row0 + nc;
    uint64_t *h_tok0 = reinterpret_cast<uint64_t *>(h_len + nc + (nc & 1));
    uint64_t *h_slot = h_tok0 + nc;
    int max_len = 0;
    h_slot[0] = 0;
    for (int i = 0; i < nc; i++) {
        h_row0[i] = (int)(starts[c0 + i] - starts[c0]);
        h_len[i] = (int)(starts[c0 + i + 1] - starts[c0 + i]);
        h_tok0[i] = (uint64_t)h_row0[i];
        h_slot[i + 1] = h_slot[i] + 4ull * (uint64_t)h_len[i] + 8ull;
        max_len = std::max(max_len, h_len[i]);
    }
    // attention CTAs (one per chunk) longest chunk first: the short chunks (document
    // tails) then fill the last round of CTAs instead of leaving SMs idle
    int *h_arow0 = reinterpret_cast<int *>(h_slot + nc + 1);
    int *h_alen = h_arow0 + nc;
    int *h_akv = h_alen + nc;
    c->att_order.resize(nc);
    for (int i = 0; i < nc; i++) c->att_order[i] = i;
    std::stable_sort(c->att_order.begin(), c->att_order.end(), [&](int a, int b) { return h_len[a] > h_len[b]; });
    for (int i = 0; i < nc; i++) {
        h_arow0[i] = h_row0[c->att_order[i]];
        h_alen[i] = h_len[c->att_order[i]];
        h_akv[i] = h_row0[c->att_order[i]] + 32 * c->att_order[i];   // k_kv_prep_split's chunk offsets
    }
    cudaMemcpyAsync(c->chunk_row0, h_row0, sizeof(int) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->chunk_len, h_len, sizeof(int) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->att_row0, h_arow0, sizeof(int) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->att_len, h_alen, sizeof(int) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->att_kvoff, h_akv, sizeof(int) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->chunk_tok0, h_tok0, sizeof(uint64_t) * nc, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(c->slot_off, h_slot, sizeof(uint64_t) * (nc + 1), cudaMemcpyHostToDevice, st);
    cudaMemsetAsync(c->err_flag, 0, sizeof(int), st);
    return max_len;
}

// Run the model + CDF + encoder for chunks [c0, c1); rows are the wave's tokens.
// d_tok: device pointer to the wave's first token.  Results stay on device.
int run_wave(czg_ctx *c, const uint32_t *d_tok, const uint64_t *starts, uint32_t c0, uint32_t c1,
             const Trace *tr) {
    const czg_model_info &m = c->info;
    const int d = m.d_model, dff = c->dff_pad, V = m.vocab_size, H = m.n_heads;
    const int nc = (int)(c1 - c0);
    const int M = (int)(starts[c1] - starts[c0]);
    cudaStream_t st = c->stream;
    const int max_len = wave_meta(c, starts, c0, c1);

    timed(c, kRows, [&] {
        launch_rows(d_tok, c->chunk_row0, c->chunk_len, c->chunk_tok0, nc, V, c->tok_in, c->tok_out,
                    c->pos, c->rowchunk, c->err_flag, st);
    });
    // the first pre-norm from the per-token table (the residual of layer 0 is re-read
    // from the embedding by the first residual norm)
    timed(c, kEmbedNorm, [&] { launch_xn_gather(c->tok_in, c->xn_tab, M, d, c->xn, st); });
    // tensor-core attention, K/V tiles streamed per warp from a per-chunk layout (at
    // 1024 keys 129.6 ms per configuration-1 step against 136.0 with the chunk's
    // K/V^T staged in shared memory, which CZG_ATTN_STAGED=1 selects up to 1024 keys)
    const bool staged = c->staged_attention && attention_mma_fits(max_len) && !c->scalar_attention;
    const bool stream = !staged && !c->scalar_attention;
    // the streamed layout's K (rotated) and V come out of the QKV GEMM's epilogue
    // (CZG_KV_EPILOGUE=0: k_kv_prep_split after a plain requantising GEMM)
    const char *kve = getenv("CZG_KV_EPILOGUE");
    const bool kv_epi = stream && !(kve && kve[0] == '0');
    KvSplit kvs;
    kvs.rowchunk = c->rowchunk;
    kvs.chunk_row0 = c->chunk_row0;
    kvs.chunk_len = c->chunk_len;
    kvs.rope_cos = c->rope_cos;
    kvs.rope_sin = c->rope_sin;
    kvs.kv = c->kv;
    kvs.d = d;
    for (int l = 0; l < m.n_layers; l++) {
        const LayerDev &L = c->layers[l];
        timed(c, kGemmQkv, [&] {
            if (kv_epi)
                gemm(c, c->tm_xn, L.tm_qkv, M, d + 128, d, kEpiRequantKv, L.qkv_mult, L.qkv_shift, c->qkv, d + 128,
                     &kvs);
            else
                gemm(c, c->tm_xn, L.tm_qkv, M, d + 128, d, kEpiRequant, L.qkv_mult, L.qkv_shift, c->qkv, d + 128);
        });
        if (!kv_epi)
            timed(c, kKvPrep, [&] {
                if (stream)
                    launch_kv_prep_split(c->qkv, d + 128, d, c->pos, c->rowchunk, c->chunk_row0, c->chunk_len,
                                         c->rope_cos, c->rope_sin, M, c->kv, st);
                else
                    launch_kv_prep(c->qkv, d + 128, d, c->pos, c->rope_cos, c->rope_sin, M, c->kv, st);
            });
        timed(c, kAttention, [&] {
            if (staged)
                launch_attention_mma(c->qkv, d + 128, c->kv, c->att_row0, c->att_len, nc, max_len, H,
                                     L.score_mult, L.sink_key, c->rope_cos, c->rope_sin, c->lut4k,
                                     L.score_mode, c->exp0, c->attn, d, st);
            else if (stream)
                launch_attention_mma_stream(c->qkv, d + 128, c->kv, c->att_row0, c->att_len, c->att_kvoff, nc,
                                            max_len, H, L.score_mult, L.sink_key, c->rope_cos, c->rope_sin,
                                            c->lut4k, L.score_mode, c->exp0, c->attn, d, c->task_ctr, st);
            else
                launch_attention(c->qkv, d + 128, c->kv, c->att_row0, c->att_len, nc, max_len, H,
                                 L.score_mult, L.sink_key, c->rope_cos, c->rope_sin, c->lut, c->attn, d, st);
        });
        if (tr && tr->attn)
            cudaMemcpy2DAsync(tr->attn + (size_t)l * d, (size_t)m.n_layers * d, c->attn, d, d, M,
                              cudaMemcpyDeviceToHost, st);
        o_norm(c, L, l, M, st);
        timed(c, kGemmUp, [&] {
            gemm(c, c->tm_xn, L.tm_up, M, 2 * dff, d, kEpiReglu, L.up_mult, L.up_shift,
                 c->hbuf, dff);
        });
        down_norm(c, L, l, M, st);
    }
    if (tr && tr->final_in)
        cudaMemcpyAsync(tr->final_in, c->xn, (size_t)M * d, cudaMemcpyDeviceToHost, st);
    bool fused = false;
    if (c->head_cdf && !tr) {   // a trace wants the logits themselves
        timed(c, kHeadCdf, [&] {
            fused = launch_head_cdf(c->tm_xn, c->tm_head, M, V, d, c->tok_out, c->lut4k, m.coef_q24 << 8,
                                    m.target_total, c->lohi, c->err_flag, st);
        });
    }
    if (!fused) {
        timed(c, kGemmHead, [&] {
            gemm(c, c->tm_xn, c->tm_head, M, c->vpad, d, kEpiInt32, 1, 0, c->logits, c->vpad);
        });
        if (tr && tr->logits)
            cudaMemcpy2DAsync(tr->logits, (size_t)V * 4, c->logits, (size_t)c->vpad * 4, (size_t)V * 4, M,
                              cudaMemcpyDeviceToHost, st);
        timed(c, kCdf, [&] {
            launch_cdf_lohi(c->logits, V, c->vpad, c->tok_out, c->lut, c->lut4k, c->exp0 && c->logit_small, m.coef_q24,
                            m.target_total, M, c->lohi, st);
        });
    }
    if (tr && tr->lohi)
        cudaMemcpyAsync(tr->lohi, c->lohi, (size_t)M * 8, cudaMemcpyDeviceToHost, st);
    timed(c, kEncode, [&] {
        launch_encode(c->lohi, c->chunk_row0, c->chunk_len, nc, m.target_total, c->slots, c->slot_off,
                      c->lens, c->err_flag, st);
    });
    if (c->gemm_failed) {
        c->gemm_failed = false;
        return fail(c, CZG_E_DEVICE, "a GEMM launch was refused (output tensor map)");
    }
    if (!cuda_ok(c, cudaGetLastError(), "kernel launch")) return CZG_E_DEVICE;
    return CZG_OK;
}

struct WavePlan {
    uint32_t c0, c1;
};

std::vector<WavePlan> plan_waves(const czg_ctx *c, const uint64_t *starts, uint32_t n) {
    std::vector<WavePlan> w;
    uint32_t c0 = 0;
    while (c0 < n) {
        uint32_t c1 = c0;
        while (c1 < n && (c1 - c0) < (uint32_t)c->cap_chunks &&
               starts[c1 + 1] - starts[c0] <= (uint64_t)c->cap_rows)
            c1++;
        w.push_back({c0, c1});
        c0 = c1;
    }
    return w;
}

void stats_begin(czg_ctx *c) {
    memset(&c->stats, 0, sizeof(c->stats));
    c->stats.n_classes = kNumClasses;
    c->ev_used = 0;
    cudaEventRecord(c->ev_begin, c->stream);
}

void stats_end(czg_ctx *c) {
    cudaEventRecord(c->ev_end, c->stream);
    cudaEventSynchronize(c->ev_end);
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev_begin, c->ev_end);
    c->stats.total_ms = ms;
}

// After a wave's encoder: the chunk lengths and the error word to the host, packed
// offsets, then pack the chunks and copy them to out + total (when they fit).
int wave_copy_out(czg_ctx *c, uint32_t c0, int nc, uint8_t *out, uint64_t out_cap, uint32_t *out_lens,
                  uint64_t &total, int &status) {
    int err = 0;
    cudaMemcpyAsync(out_lens + c0, c->lens, sizeof(uint32_t) * nc, cudaMemcpyDeviceToHost, c->stream);
    cudaMemcpyAsync(&err, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
    if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "wave")) return CZG_E_DEVICE;
    c->stats.d2h_bytes += sizeof(uint32_t) * nc;
    if (err & kErrToken) return fail(c, CZG_E_TOKEN, "token id >= vocab_size");
    if (err & kErrOverflow) return fail(c, CZG_E_DEVICE, "encoder slot overflow");
    if (err & kErrTimeout) return fail(c, CZG_E_TIMEOUT, "a bounded device wait expired");
    uint64_t *h_pack = reinterpret_cast<uint64_t *>(c->h_meta_cur);
    h_pack[0] = 0;
    for (int i = 0; i < nc; i++) h_pack[i + 1] = h_pack[i] + out_lens[c0 + i];
    const uint64_t wave_bytes = h_pack[nc];
    if (total + wave_bytes <= out_cap) {
        cudaMemcpyAsync(c->pack_off, h_pack, sizeof(uint64_t) * (nc + 1), cudaMemcpyHostToDevice, c->stream);
        timed(c, kPack, [&] { launch_pack(c->slots, c->slot_off, c->lens, c->pack_off, nc, c->packed, c->stream); });
        EvPair &e = next_ev(c, -2);
        cudaEventRecord(e.a, c->stream);
        cudaMemcpyAsync(out + total, c->packed, wave_bytes, cudaMemcpyDeviceToHost, c->stream);
        cudaEventRecord(e.b, c->stream);
        c->stats.d2h_bytes += wave_bytes;
    } else {
        status = CZG_E_CAPACITY;
    }
    total += wave_bytes;
    if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "wave copy-out")) return CZG_E_DEVICE;
    collect_events(c);
    return CZG_OK;
}

int compress_impl(czg_ctx *c, const uint32_t *tokens, bool device_tokens, const uint64_t *starts,
                  uint32_t n_chunks, uint8_t *out, uint64_t out_cap, uint32_t *out_lens,
                  uint64_t *out_needed) {
    if (!c) return CZG_E_ARG;
    if ((!starts && n_chunks) || (n_chunks && !tokens)) return fail(c, CZG_E_ARG, "null input pointer");
    uint64_t ntok = n_chunks ? starts[n_chunks] - starts[0] : 0;
    const int limit = std::min(c->info.context_length, c->info.max_seq_len);
    for (uint32_t i = 0; i < n_chunks; i++) {
        if (starts[i + 1] < starts[i]) return fail(c, CZG_E_ARG, "chunk_starts must be non-decreasing");
        if (starts[i + 1] - starts[i] > (uint64_t)limit)
            return fail(c, CZG_E_CHUNK, "chunk " + std::to_string(i) + " is longer than the model's context");
    }
    uint64_t bound = czg_compress_bound(ntok, n_chunks);
    if (!out) {
        if (out_needed) *out_needed = bound;
        return CZG_OK;
    }
    if (!out_lens) return fail(c, CZG_E_ARG, "out_lens is null");
    if (!cuda_ok(c, cudaSetDevice(c->device), "cudaSetDevice")) return CZG_E_DEVICE;
    stats_begin(c);
    c->stats.n_tokens = ntok;
    c->stats.n_chunks = n_chunks;
    if (int st = ensure_workspace(c, ntok)) return st;
    // Waves are pipelined: wave i's tokens go up on the copy stream into buffer i % 2
    // while wave i-1 computes; its chunks are packed on the device (offsets by a scan)
    // into packed buffer i % 2, and only its lengths, total and error word come back
    // before the host launches wave i+1 -- the packed bytes of wave i follow on the
    // copy stream while wave i+1 computes.
    const std::vector<WavePlan> waves = plan_waves(c, starts, n_chunks);
    uint64_t total = 0;
    int status = CZG_OK;
    auto enqueue = [&](const WavePlan &w, int b) -> int {
        const uint64_t t0 = starts[w.c0], nt = starts[w.c1] - t0;
        const int nc = (int)(w.c1 - w.c0);
        const uint32_t *d_tok = tokens + t0;
        if (!device_tokens) {
            uint32_t *buf = b ? c->tokens2 : c->tokens;
            cudaStreamWaitEvent(c->copy_stream, c->ev_comp[b], 0);   // wave i-2 has read the buffer
            EvPair &e = next_ev(c, -1);
            cudaEventRecord(e.a, c->copy_stream);
            cudaMemcpyAsync(buf, tokens + t0, nt * 4, cudaMemcpyHostToDevice, c->copy_stream);
            cudaEventRecord(e.b, c->copy_stream);
            cudaEventRecord(c->ev_h2d[b], c->copy_stream);
            cudaStreamWaitEvent(c->stream, c->ev_h2d[b], 0);
            c->stats.h2d_bytes += nt * 4;
            d_tok = buf;
        }
        c->h_meta_cur = b ? c->h_meta2 : c->h_meta;
        if (int st = run_wave(c, d_tok, starts, w.c0, w.c1, nullptr)) return st;
        uint8_t *packed = b ? c->packed2 : c->packed;
        launch_pack_offsets(c->lens, nc, c->pack_off, c->stream);
        cudaStreamWaitEvent(c->stream, c->ev_d2h[b], 0);   // wave i-2's bytes have left the buffer
        timed(c, kPack, [&] { launch_pack(c->slots, c->slot_off, c->lens, c->pack_off, nc, packed, c->stream); });
        uint8_t *hs = c->h_small[b];
        cudaMemcpyAsync(hs, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
        cudaMemcpyAsync(hs + 8, c->pack_off + nc, sizeof(uint64_t), cudaMemcpyDeviceToHost, c->stream);
        cudaMemcpyAsync(hs + 16, c->lens, sizeof(uint32_t) * nc, cudaMemcpyDeviceToHost, c->stream);
        cudaEventRecord(c->ev_small[b], c->stream);
        cudaEventRecord(c->ev_comp[b], c->stream);
        if (!cuda_ok(c, cudaGetLastError(), "wave launch")) return CZG_E_DEVICE;
        return CZG_OK;
    };
    auto finish = [&](const WavePlan &w, int b) -> int {
        const int nc = (int)(w.c1 - w.c0);
        if (!cuda_ok(c, cudaEventSynchronize(c->ev_small[b]), "wave")) return CZG_E_DEVICE;
        const uint8_t *hs = c->h_small[b];
        int err = 0;
        uint64_t wave_bytes = 0;
        memcpy(&err, hs, sizeof(int));
        memcpy(&wave_bytes, hs + 8, sizeof(uint64_t));
        memcpy(out_lens + w.c0, hs + 16, sizeof(uint32_t) * nc);
        c->stats.d2h_bytes += 12 + sizeof(uint32_t) * (uint64_t)nc;
        if (err & kErrToken) return fail(c, CZG_E_TOKEN, "token id >= vocab_size");
        if (err & kErrOverflow) return fail(c, CZG_E_DEVICE, "encoder slot overflow");
        if (err & kErrTimeout) return fail(c, CZG_E_TIMEOUT, "a bounded device wait expired");
        if (total + wave_bytes <= out_cap) {
            EvPair &e = next_ev(c, -2);
            cudaEventRecord(e.a, c->copy_stream);
            cudaMemcpyAsync(out + total, b ? c->packed2 : c->packed, wave_bytes, cudaMemcpyDeviceToHost,
                            c->copy_stream);
            cudaEventRecord(e.b, c->copy_stream);
            cudaEventRecord(c->ev_d2h[b], c->copy_stream);
            c->stats.d2h_bytes += wave_bytes;
        } else {
            status = CZG_E_CAPACITY;
        }
        total += wave_bytes;
        return CZG_OK;
    };
    int st = CZG_OK;
    for (size_t i = 0; i < waves.size() && !st; i++) {
        st = enqueue(waves[i], (int)(i & 1));
        if (!st && i >= 1) st = finish(waves[i - 1], (int)((i - 1) & 1));
    }
    if (!st && !waves.empty()) st = finish(waves.back(), (int)((waves.size() - 1) & 1));
    // the last copies complete before the call returns (and before its end event)
    const bool drained = cudaStreamSynchronize(c->copy_stream) == cudaSuccess;
    if (st) {
        cudaStreamSynchronize(c->stream);
        return st;
    }
    if (!cuda_ok(c, drained ? cudaSuccess : cudaErrorUnknown, "wave copy-out")) return CZG_E_DEVICE;
    collect_events(c);
    stats_end(c);
    if (out_needed) *out_needed = total;
    if (status == CZG_E_CAPACITY) return fail(c, CZG_E_CAPACITY, "output buffer too small");
    return CZG_OK;
}

// (Re)allocate the decompression buffers for `streams` streams of up to `len`
// positions, `bytes` chunk bytes and `tokens` output tokens.
int dec_reserve(czg_ctx *c, size_t streams, size_t len, size_t bytes, size_t tokens) {
    const int L = c->info.n_layers;
    if (streams <= c->dec_streams && len <= c->dec_len && bytes <= c->dec_bytes && tokens <= c->dec_tokens)
        return CZG_OK;
    for (void *p : c->dec_allocs) cudaFree(p);
    c->dec_allocs.clear();
    streams = std::max(streams, c->dec_streams);
    len = (std::max(len, c->dec_len) + 31) & ~(size_t)31;   // the split KV layout reads whole 32-key tiles
    bytes = std::max(bytes, c->dec_bytes);
    tokens = std::max(tokens, c->dec_tokens);
    auto get = [&](void **p, size_t n) {
        if (cudaMalloc(p, std::max<size_t>(n, 16)) != cudaSuccess) return false;
        c->dec_allocs.push_back(*p);
        return true;
    };
    bool ok = get((void **)&c->kvc, (size_t)L * streams * len * 128) &&
              get((void **)&c->dstate, streams * sizeof(DecState)) && get((void **)&c->ddata, bytes + 16) &&
              get((void **)&c->d_off, streams * 8) && get((void **)&c->d_len, streams * 8) &&
              get((void **)&c->d_tokoff, streams * 8) && get((void **)&c->d_outtok, tokens * 4 + 16);
    if (!ok) {
        for (void *p : c->dec_allocs) cudaFree(p);
        c->dec_allocs.clear();
        c->dec_streams = c->dec_len = c->dec_bytes = c->dec_tokens = 0;
        cudaGetLastError();
        return fail(c, CZG_E_DEVICE, "cudaMalloc failed for the decompression buffers");
    }
    c->dec_streams = streams;
    c->dec_len = len;
    c->dec_bytes = bytes;
    c->dec_tokens = tokens;
    return CZG_OK;
}

// n bytes of host memory copied by up to eight threads (the calling one included);
// a thread that cannot be started leaves its slices to the calling thread
void parallel_memcpy(uint8_t *dst, const uint8_t *src, size_t n) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t nt = std::max<size_t>(1, std::min<size_t>(std::min(8u, hw), n >> 22));   // >= 4 MB per thread
    const size_t per = ((n + nt - 1) / nt + 63) & ~(size_t)63;   // slices of 64-byte multiples covering n
    std::vector<std::thread> pool;
    size_t done = std::min(n, per);   // [0, done) is this thread's or a started thread's
    for (size_t i = 1; i < nt; i++) {
        const size_t a = std::min(n, i * per), b = std::min(n, a + per);
        if (a >= b) break;
        try {
            pool.emplace_back([=] { memcpy(dst + a, src + a, b - a); });
        } catch (...) {   // no thread to be had: the rest in this one
            break;
        }
        done = b;
    }
    memcpy(dst, src, std::min(n, per));
    if (done < n) memcpy(dst + done, src + done, n - done);
    for (auto &t : pool) t.join();
}

// Device memory to a caller's (pageable) host buffer: DMAs into pinned staging at
// full PCIe / C2C speed, then host threads copy it on (a direct copy to pageable
// memory goes through the driver's staging at a few GB/s).  The staging buffer is
// at most CZG_COPY_STAGING_BYTES (default 256 MB; larger results go through it in
// pieces).  Small copies, or no pinned memory to be had, take the direct copy.
// Returns false on a CUDA error.
bool copy_out(czg_ctx *c, void *dst, const void *src, size_t n, cudaStream_t s) {
    if (n == 0) return true;
    size_t cap = (size_t)256 << 20;
    if (const char *ev = getenv("CZG_COPY_STAGING_BYTES")) cap = std::max<size_t>((size_t)1 << 22, strtoull(ev, nullptr, 10));
    const size_t want = std::min(n, cap);
    if (n >= ((size_t)1 << 22) && want > c->h_out_bytes) {
        if (c->h_out) {
            cudaFreeHost(c->h_out);
            c->h_out = nullptr;
            c->h_out_bytes = 0;
        }
        if (cudaMallocHost(&c->h_out, want) == cudaSuccess) c->h_out_bytes = want;
        else { c->h_out = nullptr; cudaGetLastError(); }
    }
    if (n < ((size_t)1 << 22) || c->h_out_bytes == 0) {
        cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, s);
        return cudaStreamSynchronize(s) == cudaSuccess;
    }
    for (size_t off = 0; off < n; off += c->h_out_bytes) {
        const size_t len = std::min(c->h_out_bytes, n - off);
        cudaMemcpyAsync(c->h_out, (const uint8_t *)src + off, len, cudaMemcpyDeviceToHost, s);
        if (cudaStreamSynchronize(s) != cudaSuccess) return false;
        parallel_memcpy((uint8_t *)dst + off, c->h_out, len);
    }
    return true;
}

// Decompress: all chunks of a wave decode in lockstep, longest first, so the
// active streams at step i are a prefix of the rows.
int decompress_impl(czg_ctx *c, const uint8_t *data, const uint64_t *data_starts, const uint32_t *n_tokens,
                    uint32_t n_chunks, uint32_t *out_tokens) {
    if (!c) return CZG_E_ARG;
    if (n_chunks == 0) return CZG_OK;
    if (!data_starts || !n_tokens || !out_tokens || (!data && data_starts[n_chunks] > data_starts[0]))
        return fail(c, CZG_E_ARG, "null input pointer");
    const czg_model_info &m = c->info;
    const int d = m.d_model, dff = c->dff_pad, V = m.vocab_size, H = m.n_heads;
    const int limit = std::min(m.context_length, m.max_seq_len);
    uint64_t total_tok = 0;
    int max_len = 0;
    for (uint32_t i = 0; i < n_chunks; i++) {
        if (data_starts[i + 1] < data_starts[i]) return fail(c, CZG_E_ARG, "data_starts must be non-decreasing");
        if ((int64_t)n_tokens[i] > limit)
            return fail(c, CZG_E_CHUNK, "chunk " + std::to_string(i) + " is longer than the model's context");
        total_tok += n_tokens[i];
        max_len = std::max(max_len, (int)n_tokens[i]);
    }
    if (!cuda_ok(c, cudaSetDevice(c->device), "cudaSetDevice")) return CZG_E_DEVICE;
    stats_begin(c);
    c->stats.n_tokens = total_tok;
    c->stats.n_chunks = n_chunks;
    // stream order: longest first, stable (a counting sort: lengths are at most the context)
    std::vector<uint32_t> order(n_chunks);
    {
        std::vector<uint32_t> at((size_t)max_len + 2, 0);   // at[l]: first slot of length l
        for (uint32_t i = 0; i < n_chunks; i++) at[n_tokens[i]]++;
        uint32_t pos = 0;
        for (int l = max_len; l >= 0; l--) {
            const uint32_t k = at[l];
            at[l] = pos;
            pos += k;
        }
        for (uint32_t i = 0; i < n_chunks; i++) order[at[n_tokens[i]]++] = i;
    }
    std::vector<uint64_t> tok_base(n_chunks + 1, 0);
    for (uint32_t i = 0; i < n_chunks; i++) tok_base[i + 1] = tok_base[i] + n_tokens[i];
    // streams per wave: the activation rows and a KV-cache budget
    const size_t per_stream = (size_t)m.n_layers * std::max(1, max_len) * 128;
    size_t budget = (size_t)8 << 30;
    if (const char *ev = getenv("CZG_DECODE_KV_BYTES")) budget = std::max<size_t>(1 << 20, strtoull(ev, nullptr, 10));
    if (int st = ensure_workspace(c, std::min<size_t>(n_chunks, budget / per_stream))) return st;
    const size_t wave = std::max<size_t>(1, std::min<size_t>((size_t)c->cap_rows, budget / per_stream));
    const uint64_t all_bytes = data_starts[n_chunks] - data_starts[0];
    int st = dec_reserve(c, std::min<size_t>(wave, n_chunks), std::max(1, max_len), all_bytes, total_tok);
    if (st) return st;
    cudaStream_t s = c->stream;
    {
        EvPair &e = next_ev(c, -1);
        cudaEventRecord(e.a, s);
        if (all_bytes) cudaMemcpyAsync(c->ddata, data + data_starts[0], all_bytes, cudaMemcpyHostToDevice, s);
        cudaEventRecord(e.b, s);
        c->stats.h2d_bytes += all_bytes;
    }
    std::vector<uint64_t> h_off, h_len, h_tok;
    for (size_t w0 = 0; w0 < n_chunks; w0 += wave) {
        const size_t w1 = std::min<size_t>(n_chunks, w0 + wave);
        const int ns = (int)(w1 - w0);
        h_off.resize(ns);
        h_len.resize(ns);
        h_tok.resize(ns);
        for (int r = 0; r < ns; r++) {   // each stream's tokens go straight to its place in the caller's order
            const uint32_t ch = order[w0 + r];
            h_off[r] = data_starts[ch] - data_starts[0];
            h_len[r] = data_starts[ch + 1] - data_starts[ch];
            h_tok[r] = tok_base[ch];
        }
        cudaMemcpyAsync(c->d_off, h_off.data(), 8 * ns, cudaMemcpyHostToDevice, s);
        cudaMemcpyAsync(c->d_len, h_len.data(), 8 * ns, cudaMemcpyHostToDevice, s);
        cudaMemcpyAsync(c->d_tokoff, h_tok.data(), 8 * ns, cudaMemcpyHostToDevice, s);
        launch_dec_init(c->ddata, c->d_off, c->d_len, ns, c->dstate, c->tok_in, s);
        const int wmax = (int)n_tokens[order[w0]];
        const size_t cache_ld = (size_t)c->dec_len * 128;
        // tensor-core decode attention (heads as tile rows) over the split K / V^T cache layout
        const bool split = attention_decode_mma_ok(H) && getenv("CZG_SCALAR_DECODE") == nullptr;
        const size_t layer_ld = (size_t)c->dec_streams * cache_ld;
        int active = ns;
        // programmatic dependent launches for the step kernels: each may be scheduled
        // while its predecessor finishes and waits on the device for its results
        // (off with per-kernel events, or CZG_PDL=0)
        const char *pdl_env = getenv("CZG_PDL");
        const PdlScope pdl_scope(!c->kernel_timing && !(pdl_env && atoi(pdl_env) == 0));
        for (int step = 0; step < wmax; step++) {
            while (active > 0 && (int)n_tokens[order[w0 + active - 1]] <= step) active--;
            const int M = active;
            // later steps find their first pre-norm output written by the previous step's decoder
            if (step == 0) timed(c, kEmbedNorm, [&] { launch_xn_gather(c->tok_in, c->xn_tab, M, d, c->xn, s); });
            for (int l = 0; l < m.n_layers; l++) {
                const LayerDev &L = c->layers[l];
                int8_t *kvc = c->kvc + (size_t)l * layer_ld;
                timed(c, kGemmQkv, [&] {
                    gemm(c, c->tm_xn, L.tm_qkv, M, d + 128, d, kEpiRequant, L.qkv_mult, L.qkv_shift,
                         c->qkv, d + 128);
                });
                if (!split)   // the tensor-core decode kernel appends the step's K/V row itself
                    timed(c, kKvAppend, [&] {
                        launch_kv_append(c->qkv, d + 128, d, step, c->rope_cos, c->rope_sin, M, kvc, cache_ld, split,
                                         s);
                    });
                timed(c, kAttnDecode, [&] {
                    if (split)
                        launch_attention_decode_mma(c->qkv, d + 128, d, kvc, cache_ld, M, step, H, L.score_mult,
                                                    L.sink_key, c->rope_cos, c->rope_sin, c->lut4k, L.score_mode, c->exp0,
                                                    c->attn, d, s);
                    else
                        launch_attention_decode(c->qkv, d + 128, kvc, cache_ld, M, step, H, L.score_mult, L.sink_key,
                                                c->rope_cos, c->rope_sin, c->lut, c->attn, d, s);
                });
                o_norm(c, L, l, M, s);
                timed(c, kGemmUp, [&] {
                    gemm(c, c->tm_xn, L.tm_up, M, 2 * dff, d, kEpiReglu, L.up_mult, L.up_shift,
                         c->hbuf, dff);
                });
                down_norm(c, L, l, M, s);
            }
            timed(c, kGemmHead, [&] {
                gemm(c, c->tm_xn, c->tm_head, M, c->vpad, d, kEpiInt32, 1, 0, c->logits, c->vpad);
            });
            timed(c, kCdfDecode, [&] {
                launch_cdf_decode(c->logits, V, c->vpad, c->lut, c->lut4k, c->exp0 && c->logit_small, m.coef_q24, m.target_total, M, c->dstate, c->ddata,
                                  c->d_off, c->d_len, c->d_tokoff, step, c->d_outtok, c->tok_in, c->xn_tab,
                                  step + 1 < wmax ? c->xn : nullptr, d, s);
            });
            if (c->ev_used > 4096) {   // keep the event pool bounded on long chunks
                if (!cuda_ok(c, cudaStreamSynchronize(s), "decode step")) return CZG_E_DEVICE;
                collect_events(c);
            }
        }
        if (c->gemm_failed) {
            c->gemm_failed = false;
            return fail(c, CZG_E_DEVICE, "a GEMM launch was refused (output tensor map)");
        }
        if (!cuda_ok(c, cudaGetLastError(), "kernel launch")) return CZG_E_DEVICE;
        if (w1 < n_chunks) {   // the next wave reuses the per-stream buffers: end this one
            int err = 0;
            cudaMemcpyAsync(&err, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost, s);
            if (!cuda_ok(c, cudaStreamSynchronize(s), "decode wave")) return CZG_E_DEVICE;
            collect_events(c);
            if (err & kErrTimeout) return fail(c, CZG_E_TIMEOUT, "a bounded device wait expired");
        }
    }
    // every token is in caller order on the device: one copy
    {
        int err = 0;
        cudaMemcpyAsync(&err, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost, s);
        EvPair &e = next_ev(c, -2);
        cudaEventRecord(e.a, s);
        const bool ok = copy_out(c, out_tokens, c->d_outtok, total_tok * 4, s);
        cudaEventRecord(e.b, s);
        if (!ok || !cuda_ok(c, cudaStreamSynchronize(s), "decode")) return CZG_E_DEVICE;
        collect_events(c);
        c->stats.d2h_bytes += total_tok * 4;
        if (err & kErrTimeout) return fail(c, CZG_E_TIMEOUT, "a bounded device wait expired");
    }
    stats_end(c);
    return CZG_OK;
}

}  // namespace

// ---- C ABI ------------------------------------------------------------------

extern "C" {

int czg_ctx_create(int device, const uint8_t *czm, size_t czm_len, czg_ctx **out) {
    if (!out || !czm) return fail(nullptr, CZG_E_ARG, "null argument");
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return fail(nullptr, CZG_E_DEVICE, "no such CUDA device");
    czg_ctx *c = new czg_ctx();
    c->device = device;
    int st = CZG_OK;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        st = fail(c, CZG_E_DEVICE, "cannot initialise the device");
    }
    c->stream = c->own_stream;
    if (!st) st = load_model(c, czm, czm_len);
    c->scalar_attention = getenv("CZG_SCALAR_ATTENTION") && atoi(getenv("CZG_SCALAR_ATTENTION")) != 0;
    c->staged_attention = getenv("CZG_ATTN_STAGED") && atoi(getenv("CZG_ATTN_STAGED")) != 0;
    c->kernel_timing = getenv("CZG_KERNEL_TIMING") && atoi(getenv("CZG_KERNEL_TIMING")) != 0;
    // tokens per wave: large waves keep every SM busy through the per-chunk serial
    // encoder and the attention's last CTAs; the workspace grows to it on demand
    int wave = 1 << 22;
    if (const char *e = getenv("CZG_WAVE_TOKENS")) wave = std::max(16384, atoi(e));
    c->wave_cap = wave;
    if (!st) st = alloc_workspace(c, std::min(wave, 1 << 16), std::max(1024, std::min(wave, 1 << 16) / 16));
    if (!st) {
        cudaEventCreate(&c->ev_begin);
        cudaEventCreate(&c->ev_end);
        bool ok = cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) == cudaSuccess;
        for (int b = 0; b < 2 && ok; b++)
            for (cudaEvent_t *e : {&c->ev_h2d[b], &c->ev_comp[b], &c->ev_small[b], &c->ev_d2h[b]})
                ok = ok && cudaEventCreateWithFlags(e, cudaEventDisableTiming) == cudaSuccess;
        if (!ok) st = fail(c, CZG_E_DEVICE, "cannot create the copy stream and its events");
        kernels_init();
        if (!cuda_ok(c, cudaDeviceSynchronize(), "init")) st = CZG_E_DEVICE;
    }
    if (st) {
        g_create_error = c->err;
        czg_ctx_destroy(c);
        return st;
    }
    *out = c;
    return CZG_OK;
}

void czg_ctx_destroy(czg_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->own_stream && c->own_stream != c->stream) cudaStreamSynchronize(c->own_stream);
    for (void *p : c->allocs) cudaFree(p);
    for (void *p : c->ws_allocs) cudaFree(p);
    for (void *p : c->dec_allocs) cudaFree(p);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    for (uint8_t *h : {c->h_meta, c->h_meta2, c->h_small[0], c->h_small[1], c->h_out})
        if (h) cudaFreeHost(h);
    for (int b = 0; b < 2; b++)
        for (cudaEvent_t e : {c->ev_h2d[b], c->ev_comp[b], c->ev_small[b], c->ev_d2h[b]})
            if (e) cudaEventDestroy(e);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    for (auto &e : c->evs) { cudaEventDestroy(e.a); cudaEventDestroy(e.b); }
    if (c->ev_begin) cudaEventDestroy(c->ev_begin);
    if (c->ev_end) cudaEventDestroy(c->ev_end);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

const char *czg_last_error(const czg_ctx *c) { return c ? c->err.c_str() : g_create_error.c_str(); }

int czg_model_info_get(const czg_ctx *c, czg_model_info *out) {
    if (!c || !out) return CZG_E_ARG;
    *out = c->info;
    return CZG_OK;
}

uint64_t czg_compress_bound(uint64_t n_tokens, uint64_t n_chunks) { return 4 * n_tokens + 8 * n_chunks; }

int czg_compress_chunks(czg_ctx *c, const uint32_t *tokens, const uint64_t *starts, uint32_t n_chunks,
                        uint8_t *out, uint64_t out_cap, uint32_t *out_lens, uint64_t *out_needed) {
    return compress_impl(c, tokens, false, starts, n_chunks, out, out_cap, out_lens, out_needed);
}

int czg_compress_chunks_device(czg_ctx *c, const uint32_t *d_tokens, const uint64_t *starts,
                               uint32_t n_chunks, uint8_t *out, uint64_t out_cap, uint32_t *out_lens,
                               uint64_t *out_needed) {
    return compress_impl(c, d_tokens, true, starts, n_chunks, out, out_cap, out_lens, out_needed);
}

int czg_decompress_chunks(czg_ctx *c, const uint8_t *data, const uint64_t *data_starts, const uint32_t *n_tokens,
                          uint32_t n_chunks, uint32_t *out_tokens) {
    return decompress_impl(c, data, data_starts, n_tokens, n_chunks, out_tokens);
}

int czg_set_stream(czg_ctx *c, void *stream) {
    if (!c) return CZG_E_ARG;
    if (!cuda_ok(c, cudaSetDevice(c->device), "cudaSetDevice")) return CZG_E_DEVICE;
    if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "cudaStreamSynchronize")) return CZG_E_DEVICE;
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return CZG_OK;
}

int czg_set_kernel_timing(czg_ctx *c, int on) {
    if (!c) return CZG_E_ARG;
    c->kernel_timing = on != 0;
    return CZG_OK;
}

int czg_last_stats(const czg_ctx *c, czg_stats *out) {
    if (!c || !out) return CZG_E_ARG;
    *out = c->stats;
    return CZG_OK;
}

const char *czg_kernel_name(uint32_t k) { return k < kNumClasses ? kClassNames[k] : ""; }

int czg_debug_trace(czg_ctx *c, const uint32_t *tokens, uint32_t n, int32_t *logits, uint32_t *lohi,
                    int8_t *attn, int8_t *final_in) {
    if (!c || (!tokens && n)) return CZG_E_ARG;
    const int limit = std::min(c->info.context_length, c->info.max_seq_len);
    if ((int64_t)n > limit) return fail(c, CZG_E_CHUNK, "chunk longer than the model's context");
    if (n == 0) return CZG_OK;
    if (!cuda_ok(c, cudaSetDevice(c->device), "cudaSetDevice")) return CZG_E_DEVICE;
    stats_begin(c);
    uint64_t starts[2] = {0, n};
    cudaMemcpyAsync(c->tokens, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream);
    Trace tr{logits, lohi, attn, final_in};
    int st = run_wave(c, c->tokens, starts, 0, 1, &tr);
    if (st) return st;
    int err = 0;
    cudaMemcpyAsync(&err, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost, c->stream);
    if (!cuda_ok(c, cudaStreamSynchronize(c->stream), "trace")) return CZG_E_DEVICE;
    collect_events(c);
    stats_end(c);
    if (err & kErrToken) return fail(c, CZG_E_TOKEN, "token id >= vocab_size");
    if (err & kErrTimeout) return fail(c, CZG_E_TIMEOUT, "a bounded device wait expired");
    return CZG_OK;
}

int czg_debug_encode_intervals(czg_ctx *c, const uint32_t *lohi, const uint64_t *starts, uint32_t n_chunks,
                               uint8_t *out, uint64_t out_cap, uint32_t *out_lens, uint64_t *out_needed) {
    if (!c) return CZG_E_ARG;
    if ((!starts && n_chunks) || (n_chunks && !lohi)) return fail(c, CZG_E_ARG, "null input pointer");
    for (uint32_t i = 0; i < n_chunks; i++)
        if (starts[i + 1] < starts[i]) return fail(c, CZG_E_ARG, "chunk_starts must be non-decreasing");
    const uint64_t ntok = n_chunks ? starts[n_chunks] - starts[0] : 0;
    if (!out) {
        if (out_needed) *out_needed = czg_compress_bound(ntok, n_chunks);
        return CZG_OK;
    }
    if (!out_lens) return fail(c, CZG_E_ARG, "out_lens is null");
    if (!cuda_ok(c, cudaSetDevice(c->device), "cudaSetDevice")) return CZG_E_DEVICE;
    stats_begin(c);
    if (int st = ensure_workspace(c, ntok)) return st;
    uint64_t total = 0;
    int status = CZG_OK;
    for (const WavePlan &w : plan_waves(c, starts, n_chunks)) {
        const uint64_t t0 = starts[w.c0], nt = starts[w.c1] - t0;
        wave_meta(c, starts, w.c0, w.c1);
        cudaMemcpyAsync(c->lohi, lohi + 2 * (t0 - starts[0]), nt * 8, cudaMemcpyHostToDevice, c->stream);
        timed(c, kEncode, [&] {
            launch_encode(c->lohi, c->chunk_row0, c->chunk_len, (int)(w.c1 - w.c0), c->info.target_total, c->slots,
                          c->slot_off, c->lens, c->err_flag, c->stream);
        });
        if (!cuda_ok(c, cudaGetLastError(), "kernel launch")) return CZG_E_DEVICE;
        if (int st = wave_copy_out(c, w.c0, (int)(w.c1 - w.c0), out, out_cap, out_lens, total, status)) return st;
    }
    stats_end(c);
    if (out_needed) *out_needed = total;
    if (status == CZG_E_CAPACITY) return fail(c, CZG_E_CAPACITY, "output buffer too small");
    return CZG_OK;
}

}  // extern "C"
