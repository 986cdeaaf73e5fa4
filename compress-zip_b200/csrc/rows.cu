// rows.cu -- per-token row kernels: row set-up, embedding + RMSNorm, and the
// fused "post-norm, residual add, next pre-norm" step that follows the O and
// down projections.  One warp per token row; d_model must be a multiple of 128.
// The residual stream is int32 in the reference; every addend is a norm output
// (|y| <= 127) and the start an embedding byte, so |x| <= 128 + 254 * n_layers
// and int16 storage is exact for n_layers <= 128 (RT = int16_t), halving its traffic.
//
// Reference: the residual stream and sandwich norms of rust/src/model.rs:362-480,
// RMSNorm of rust/src/rmsnorm.rs:40-75.
#include "common.cuh"
#include "kernels.h"

namespace czg {

// One CTA per chunk: token ids into the forward (BOS at position 0, else the
// previous token, rust/src/main.rs:212-214), the symbol to encode, the position,
// and the row's chunk.
__global__ void k_rows(const uint32_t *__restrict__ tokens, const int *__restrict__ chunk_row0,
                       const int *__restrict__ chunk_len, const uint64_t *__restrict__ chunk_tok0,
                       int vocab, uint32_t *__restrict__ tok_in, uint32_t *__restrict__ tok_out,
                       int *__restrict__ pos, int *__restrict__ rowchunk, int *__restrict__ err) {
    int c = blockIdx.x;
    int r0 = chunk_row0[c], n = chunk_len[c];
    const uint32_t *src = tokens + chunk_tok0[c];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        uint32_t t = src[i];
        uint32_t prev = i == 0 ? kBos : src[i - 1];
        if (t >= (uint32_t)vocab) atomicOr(err, kErrToken);
        tok_in[r0 + i] = min(prev, (uint32_t)(vocab - 1));   // kept in bounds; the error flag reports it
        tok_out[r0 + i] = min(t, (uint32_t)(vocab - 1));
        pos[r0 + i] = i;
        rowchunk[r0 + i] = c;
    }
}

// inv_rms_q15 by floor(sum_sq / d): every norm input is clamped to +-127, so the
// mean square is at most 127^2 (rmsnorm.rs:14-30 with the model's eps folded in).
constexpr int kInvTab = kInvTabEntries;
__global__ void k_inv_table(int eps, uint16_t *__restrict__ tab) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < kInvTab) tab[m] = (uint16_t)inv_rms_q15((uint32_t)m, 1, eps);   // floor(m / 1) + eps
}

// Warp-level RMSNorm of one row held as D/128 words of 4 int8 per lane
// (lane owns bytes [4*lane + 128*j, +4)).  rmsnorm.rs:40-75.  The sum of squares
// uses dp4a (exact: at most 4 * 127^2 per call); round_even(t / 2^15) is
// (t + 2^14 - 1 + ((t >> 15) & 1)) >> 15, exact for |t| <= 127 * 127 * 2^15.
template <int NW>
__device__ __forceinline__ void rmsnorm_words(const uint32_t (&x)[NW], const uint32_t (&w)[NW],
                                              const uint16_t *__restrict__ inv_tab, uint32_t (&y)[NW]) {
    constexpr int D = NW * 128;
    int ss = 0;
#pragma unroll
    for (int j = 0; j < NW; j++) ss = __dp4a((int)x[j], (int)x[j], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int inv = __ldg(inv_tab + min((uint32_t)ss / (uint32_t)D, (uint32_t)kInvTab - 1u));
#pragma unroll
    for (int j = 0; j < NW; j++) {
        int o4[4];
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int t = (sext8(x[j], b) * sext8(w[j], b)) * inv;
            o4[b] = clamp127((t + 0x3FFF + ((t >> 15) & 1)) >> 15);
        }
        y[j] = __byte_perm(__byte_perm(o4[0], o4[1], 0x0040), __byte_perm(o4[2], o4[3], 0x0040), 0x5410);
    }
}

// four consecutive residual elements
__device__ __forceinline__ int4 load_res4(const int32_t *p) { return *reinterpret_cast<const int4 *>(p); }
__device__ __forceinline__ int4 load_res4(const int16_t *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    return make_int4((int)(int16_t)(u.x & 0xFFFFu), (int)(int16_t)(u.x >> 16), (int)(int16_t)(u.y & 0xFFFFu),
                     (int)(int16_t)(u.y >> 16));
}
__device__ __forceinline__ void store_res4(int32_t *p, int4 v) { *reinterpret_cast<int4 *>(p) = v; }
__device__ __forceinline__ void store_res4(int16_t *p, int4 v) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(((uint32_t)v.x & 0xFFFFu) | ((uint32_t)v.y << 16),
                                               ((uint32_t)v.z & 0xFFFFu) | ((uint32_t)v.w << 16));
}

// x_res[r] = embed[tok_in[r]] (residual), xn[r] = norm(clamp(x_res[r])).  STORE
// false: the residual is not written (the first residual norm then reads the
// embedding row again, which stays in L2, instead of x_res from HBM).
template <int NW, typename RT, bool STORE>
__global__ void k_embed_norm(const uint32_t *__restrict__ tok_in, const int8_t *__restrict__ embed,
                             const int8_t *__restrict__ norm_w, int M, const uint16_t *__restrict__ inv_tab,
                             RT *__restrict__ x_res, int8_t *__restrict__ xn) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = NW * 128;
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const uint32_t *e = reinterpret_cast<const uint32_t *>(embed + (size_t)tok_in[warp] * D);
    const uint32_t *wv = reinterpret_cast<const uint32_t *>(norm_w);
    uint32_t x[NW], w[NW], y[NW];
#pragma unroll
    for (int j = 0; j < NW; j++) {
        x[j] = __ldg(e + lane + 32 * j);
        w[j] = __ldg(wv + lane + 32 * j);
    }
    if (STORE) {
        RT *xr = x_res + (size_t)warp * D;
#pragma unroll
        for (int j = 0; j < NW; j++)
            store_res4(xr + 4 * (lane + 32 * j),
                       make_int4(sext8(x[j], 0), sext8(x[j], 1), sext8(x[j], 2), sext8(x[j], 3)));
    }
#pragma unroll
    for (int j = 0; j < NW; j++) {   // clamp_i8 before the norm: -128 becomes -127
        uint32_t c = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) c |= (uint32_t)(uint8_t)clamp127(sext8(x[j], b)) << (8 * b);
        x[j] = c;
    }
    rmsnorm_words<NW>(x, w, inv_tab, y);
    uint32_t *yo = reinterpret_cast<uint32_t *>(xn + (size_t)warp * D);
#pragma unroll
    for (int j = 0; j < NW; j++) yo[lane + 32 * j] = y[j];
}

// o_n = norm(o, post_w); x_res += o_n (int32, never clamped: model.rs:432-434);
// xn = norm(clamp(x_res), next_w).  Where the residual comes from and goes (MODE):
// kResFromRes: read x_res, write it back; kResFromEmbed: the residual is still the
// embedding row of tok_in (the first norm of layer 0), written to x_res;
// kResNoStore: read x_res, write nothing back (the last norm of the model: nothing
// reads the residual afterwards).
enum { kResFromRes = 0, kResFromEmbed = 1, kResNoStore = 2 };

template <int NW, typename RT, int MODE>
__global__ void k_residual_norm(const int8_t *__restrict__ o, const int8_t *__restrict__ post_w,
                                const int8_t *__restrict__ next_w, int M, const uint16_t *__restrict__ inv_tab,
                                const uint32_t *__restrict__ tok_in, const int8_t *__restrict__ embed,
                                RT *__restrict__ x_res, int8_t *__restrict__ xn) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = NW * 128;
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const uint32_t *ov = reinterpret_cast<const uint32_t *>(o + (size_t)warp * D);
    const uint32_t *pw = reinterpret_cast<const uint32_t *>(post_w);
    const uint32_t *nw = reinterpret_cast<const uint32_t *>(next_w);
    uint32_t x[NW], w[NW], y[NW], w2[NW];
    RT *xr = x_res + (size_t)warp * D;
    const uint32_t *er = MODE == kResFromEmbed ? reinterpret_cast<const uint32_t *>(embed + (size_t)tok_in[warp] * D)
                                               : nullptr;
    int4 rv[NW];
#pragma unroll
    for (int j = 0; j < NW; j++) {   // every load of the row first
        x[j] = ov[lane + 32 * j];
        w[j] = __ldg(pw + lane + 32 * j);
        w2[j] = __ldg(nw + lane + 32 * j);
        if (MODE == kResFromEmbed) {
            const uint32_t ev = __ldg(er + lane + 32 * j);
            rv[j] = make_int4(sext8(ev, 0), sext8(ev, 1), sext8(ev, 2), sext8(ev, 3));
        } else {
            rv[j] = load_res4(xr + 4 * (lane + 32 * j));
        }
    }
    rmsnorm_words<NW>(x, w, inv_tab, y);
#pragma unroll
    for (int j = 0; j < NW; j++) {
        int4 r = rv[j];
        r.x = (int)((uint32_t)r.x + (uint32_t)sext8(y[j], 0));
        r.y = (int)((uint32_t)r.y + (uint32_t)sext8(y[j], 1));
        r.z = (int)((uint32_t)r.z + (uint32_t)sext8(y[j], 2));
        r.w = (int)((uint32_t)r.w + (uint32_t)sext8(y[j], 3));
        if (MODE != kResNoStore) store_res4(xr + 4 * (lane + 32 * j), r);
        x[j] = (uint32_t)(uint8_t)clamp127(r.x) | ((uint32_t)(uint8_t)clamp127(r.y) << 8) |
               ((uint32_t)(uint8_t)clamp127(r.z) << 16) | ((uint32_t)(uint8_t)clamp127(r.w) << 24);
    }
    rmsnorm_words<NW>(x, w2, inv_tab, y);
    uint32_t *yo = reinterpret_cast<uint32_t *>(xn + (size_t)warp * D);
#pragma unroll
    for (int j = 0; j < NW; j++) yo[lane + 32 * j] = y[j];
}

// K rotated with RoPE at the row's position and V copied, into kv[row] =
// [k_rot (64) | v (64)].  The reference reads K at qkv[d..d+64) and V at
// qkv[d+64..d+128) whatever n_kv_heads is (rust/src/attention.rs:174-194).
__global__ void k_kv_prep(const int8_t *__restrict__ qkv, int ldq, int d, const int *__restrict__ pos,
                          const int16_t *__restrict__ rope_cos, const int16_t *__restrict__ rope_sin,
                          int M, int8_t *__restrict__ kv) {
    int gid = blockIdx.x * blockDim.x + threadIdx.x;
    int row = gid >> 5, i = gid & 31;
    if (row >= M) return;
    const int8_t *k = qkv + (size_t)row * ldq + d;
    int p = pos[row];
    int x = k[i], y = k[i + kHalfDim];
    int c = rope_cos[p * kHalfDim + i], s = rope_sin[p * kHalfDim + i];
    int8_t *dst = kv + (size_t)row * 128;
    dst[i] = (int8_t)clamp127(sra_rne32(x * c - y * s, 15));            // attention.rs:29-50
    dst[i + kHalfDim] = (int8_t)clamp127(sra_rne32(x * s + y * c, 15));
    reinterpret_cast<uint16_t *>(dst + 64)[i] = reinterpret_cast<const uint16_t *>(k + 64)[i];
}

// K rotated (attention.rs:29-50) and V of every row into its chunk's streaming
// layout (the tensor-core attention for chunks longer than its shared memory
// holds): chunk c at kv + (chunk_row0[c] + 32 c) * 128 bytes, its keys' K rows of
// 64 permuted dims (bytes [16t' + 4k + b] = dim 16k + 4t' + b) first, then V in
// 32-key tiles of 2 KB from npad * 64 on (npad = len rounded up to 32), byte
// (key, dim) at tile * 2048 + (key % 32 / 4) * 256 + dim * 4 + key % 4 -- the
// decode cache layout of k_kv_append, per chunk.  One warp per row.
__global__ void k_kv_prep_split(const int8_t *__restrict__ qkv, int ldq, int d, const int *__restrict__ pos,
                                const int *__restrict__ rowchunk, const int *__restrict__ chunk_row0,
                                const int *__restrict__ chunk_len, const int16_t *__restrict__ rope_cos,
                                const int16_t *__restrict__ rope_sin, int M, int8_t *__restrict__ kv) {
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = gid >> 5, i = gid & 31;
    if (row >= M) return;
    const int8_t *k = qkv + (size_t)row * ldq + d;
    const int p = pos[row], c = rowchunk[row];
    const int npad = (chunk_len[c] + 31) & ~31;
    int8_t *base = kv + ((size_t)chunk_row0[c] + 32 * (size_t)c) * 128;
    const int x = k[i], y = k[i + kHalfDim];
    const int cs = rope_cos[p * kHalfDim + i], sn = rope_sin[p * kHalfDim + i];
    int8_t *kr = base + (size_t)p * 64;
    const int i2 = i + kHalfDim;
    kr[16 * ((i >> 2) & 3) + 4 * (i >> 4) + (i & 3)] = (int8_t)clamp127(sra_rne32(x * cs - y * sn, 15));
    kr[16 * ((i2 >> 2) & 3) + 4 * (i2 >> 4) + (i2 & 3)] = (int8_t)clamp127(sra_rne32(x * sn + y * cs, 15));
    int8_t *vt = base + (size_t)npad * 64 + (size_t)(p >> 5) * 2048 + ((p & 31) >> 2) * 256 + (p & 3);
    vt[(2 * i) * 4] = k[64 + 2 * i];
    vt[(2 * i + 1) * 4] = k[64 + 2 * i + 1];
}

// ---- host launchers -------------------------------------------------------

void launch_rows(const uint32_t *tokens, const int *chunk_row0, const int *chunk_len,
                 const uint64_t *chunk_tok0, int n_chunks, int vocab, uint32_t *tok_in,
                 uint32_t *tok_out, int *pos, int *rowchunk, int *err, cudaStream_t st) {
    if (n_chunks == 0) return;
    k_rows<<<n_chunks, 256, 0, st>>>(tokens, chunk_row0, chunk_len, chunk_tok0, vocab, tok_in,
                                     tok_out, pos, rowchunk, err);
}

template <typename RT, bool STORE>
void embed_norm_t(const uint32_t *tok_in, const int8_t *embed, const int8_t *norm_w, int M, int d, const uint16_t *inv_tab,
                  RT *x_res, int8_t *xn, cudaStream_t st) {
    const int blocks = (M + 7) / 8;
    switch (d / 128) {
        case 2: launch_k(k_embed_norm<2, RT, STORE>, blocks, 256, 0, st, tok_in, embed, norm_w, M, inv_tab, x_res, xn); break;
        case 3: launch_k(k_embed_norm<3, RT, STORE>, blocks, 256, 0, st, tok_in, embed, norm_w, M, inv_tab, x_res, xn); break;
        case 4: launch_k(k_embed_norm<4, RT, STORE>, blocks, 256, 0, st, tok_in, embed, norm_w, M, inv_tab, x_res, xn); break;
        default: break;
    }
}

template <typename RT, int MODE>
void residual_norm_t(const int8_t *o, const int8_t *post_w, const int8_t *next_w, int M, int d, const uint16_t *inv_tab,
                     const uint32_t *tok_in, const int8_t *embed, RT *x_res, int8_t *xn, cudaStream_t st) {
    const int blocks = (M + 7) / 8;
    switch (d / 128) {
        case 2: launch_k(k_residual_norm<2, RT, MODE>, blocks, 256, 0, st, o, post_w, next_w, M, inv_tab, tok_in, embed, x_res, xn); break;
        case 3: launch_k(k_residual_norm<3, RT, MODE>, blocks, 256, 0, st, o, post_w, next_w, M, inv_tab, tok_in, embed, x_res, xn); break;
        case 4: launch_k(k_residual_norm<4, RT, MODE>, blocks, 256, 0, st, o, post_w, next_w, M, inv_tab, tok_in, embed, x_res, xn); break;
        default: break;
    }
}

template <typename RT>
void residual_norm_mode(const int8_t *o, const int8_t *post_w, const int8_t *next_w, int M, int d,
                        const uint16_t *inv_tab, const uint32_t *tok_in, const int8_t *embed, bool store_res,
                        RT *x_res, int8_t *xn, cudaStream_t st) {
    if (embed != nullptr)
        residual_norm_t<RT, kResFromEmbed>(o, post_w, next_w, M, d, inv_tab, tok_in, embed, x_res, xn, st);
    else if (store_res)
        residual_norm_t<RT, kResFromRes>(o, post_w, next_w, M, d, inv_tab, tok_in, embed, x_res, xn, st);
    else
        residual_norm_t<RT, kResNoStore>(o, post_w, next_w, M, d, inv_tab, tok_in, embed, x_res, xn, st);
}

void launch_inv_table(int eps, uint16_t *tab, cudaStream_t st) {
    k_inv_table<<<kInvTab / 256, 256, 0, st>>>(eps, tab);
}

void launch_embed_norm(const uint32_t *tok_in, const int8_t *embed, const int8_t *norm_w, int M,
                       int d, const uint16_t *inv_tab, void *x_res, bool res16, bool store_res, int8_t *xn,
                       cudaStream_t st) {
    if (M == 0) return;
    if (res16) {
        if (store_res) embed_norm_t<int16_t, true>(tok_in, embed, norm_w, M, d, inv_tab, static_cast<int16_t *>(x_res), xn, st);
        else embed_norm_t<int16_t, false>(tok_in, embed, norm_w, M, d, inv_tab, static_cast<int16_t *>(x_res), xn, st);
    } else {
        if (store_res) embed_norm_t<int32_t, true>(tok_in, embed, norm_w, M, d, inv_tab, static_cast<int32_t *>(x_res), xn, st);
        else embed_norm_t<int32_t, false>(tok_in, embed, norm_w, M, d, inv_tab, static_cast<int32_t *>(x_res), xn, st);
    }
}

void launch_residual_norm(const int8_t *o, const int8_t *post_w, const int8_t *next_w, int M, int d,
                          const uint16_t *inv_tab, const uint32_t *tok_in, const int8_t *embed, bool store_res,
                          void *x_res, bool res16, int8_t *xn, cudaStream_t st) {
    if (M == 0) return;
    if (res16)
        residual_norm_mode(o, post_w, next_w, M, d, inv_tab, tok_in, embed, store_res, static_cast<int16_t *>(x_res), xn, st);
    else
        residual_norm_mode(o, post_w, next_w, M, d, inv_tab, tok_in, embed, store_res, static_cast<int32_t *>(x_res), xn, st);
}

void launch_kv_prep_split(const int8_t *qkv, int ldq, int d, const int *pos, const int *rowchunk,
                          const int *chunk_row0, const int *chunk_len, const int16_t *rope_cos,
                          const int16_t *rope_sin, int M, int8_t *kv, cudaStream_t st) {
    if (M == 0) return;
    const long long threads = (long long)M * 32;
    k_kv_prep_split<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(qkv, ldq, d, pos, rowchunk, chunk_row0,
                                                                       chunk_len, rope_cos, rope_sin, M, kv);
}

void launch_kv_prep(const int8_t *qkv, int ldq, int d, const int *pos, const int16_t *rope_cos,
                    const int16_t *rope_sin, int M, int8_t *kv, cudaStream_t st) {
    if (M == 0) return;
    long long threads = (long long)M * 32;
    k_kv_prep<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(qkv, ldq, d, pos, rope_cos, rope_sin,
                                                                 M, kv);
}

}  // namespace czg
