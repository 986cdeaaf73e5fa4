// rows.cu -- per-token row kernels: row set-up, embedding + RMSNorm, and the
// fused "post-norm, residual add, next pre-norm" step that follows the O and
// down projections.  One warp per token row; d_model must be a multiple of 128.
// The residual stream is int32 in the reference; every addend is a norm output
// (|y| <= 127) and the start an embedding byte, so |x| <= 128 + 254 * n_layers
// and int16 storage is exact for n_layers <= 128 (RT = int16_t), halving its traffic.
//
// Reference: the residual stream and sandwich norms of rust/src/model.rs:362-480,
// RMSNorm of rust/src/rmsnorm.rs:40-75.
#include <algorithm>

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

// RMSNorm of rmsnorm.rs:40-75, y = clamp(round_half_even(x * w * inv / 2^15), +-127)
// with inv = inv_rms_q15 of the row (table by floor(sum_sq / d)), in exact FP32
// (common.cuh, kM1Bits): IMAD gives the bits of M1 + x * w (|x * w| <= 127^2), and
// fma(M1 + x * w, inv / 2^15, M1 - 384 inv) = M1 + rne(x * w * inv / 2^15), since
// M1 * inv / 2^15 = 384 inv and inv / 2^15, M1 - 384 inv are exact floats; the clamp
// is taken on the biased bits, whose low byte is the int8 result.
struct NormRow {
    float mf, c;   // inv / 2^15, M1 - 384 inv
};
__device__ __forceinline__ NormRow norm_row(int sum_sq, int D, const uint16_t *__restrict__ inv_tab) {
    const int inv = __ldg(inv_tab + min((uint32_t)sum_sq / (uint32_t)D, (uint32_t)kInvTabEntries - 1u));
    return NormRow{__int2float_rn(inv) * (1.0f / 32768.0f), __int2float_rn(12582912 - 384 * inv)};
}
// biased bits of the clamped norm output of x (an int8 value) with weight w
__device__ __forceinline__ int norm_b(int x, int w, const NormRow &n) {
    const float pb = __int_as_float(x * w + (int)kM1Bits);
    const int yb = __float_as_int(__fmaf_rn(pb, n.mf, n.c));
    return min(max(yb, (int)kM1Bits - 127), (int)kM1Bits + 127);
}
__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// the low bytes of four biased results as one word of int8
__device__ __forceinline__ uint32_t pack_low4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
// the four int8 of a word, sign-extended: prmt's default mode copies byte b into byte 0
// (selector nibble b) and the sign of byte b into bytes 1..3 (nibbles 8 | b)
__device__ __forceinline__ void unpack4(uint32_t w, int (&v)[4]) {
    uint32_t r0, r1, r2, r3;
    asm("prmt.b32 %0, %1, 0, 0x8880;" : "=r"(r0) : "r"(w));
    asm("prmt.b32 %0, %1, 0, 0x9991;" : "=r"(r1) : "r"(w));
    asm("prmt.b32 %0, %1, 0, 0xAAA2;" : "=r"(r2) : "r"(w));
    asm("prmt.b32 %0, %1, 0, 0xBBB3;" : "=r"(r3) : "r"(w));
    v[0] = (int)r0;
    v[1] = (int)r1;
    v[2] = (int)r2;
    v[3] = (int)r3;
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

// Persistent warps walk the rows (warp w takes rows w, w + W, ...), so each warp
// unpacks its norm weights once.  A lane owns elements [4*lane + 128*j, +4).
__device__ __forceinline__ int row_warps() { return (int)(gridDim.x * blockDim.x) >> 5; }

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
    const int lane = threadIdx.x & 31;
    const uint32_t *wv = reinterpret_cast<const uint32_t *>(norm_w);
    int w[NW][4];
#pragma unroll
    for (int j = 0; j < NW; j++) unpack4(__ldg(wv + lane + 32 * j), w[j]);
    for (int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); row < M; row += row_warps()) {
        const uint32_t *e = reinterpret_cast<const uint32_t *>(embed + (size_t)tok_in[row] * D);
        int x[NW][4];
        int ss = 0;
#pragma unroll
        for (int j = 0; j < NW; j++) {
            unpack4(__ldg(e + lane + 32 * j), x[j]);
            if (STORE) store_res4(x_res + (size_t)row * D + 4 * (lane + 32 * j), make_int4(x[j][0], x[j][1], x[j][2], x[j][3]));
#pragma unroll
            for (int b = 0; b < 4; b++) {
                x[j][b] = max(x[j][b], -127);   // clamp_i8 before the norm: -128 becomes -127
                ss += x[j][b] * x[j][b];
            }
        }
        const NormRow nr = norm_row(warp_sum(ss), D, inv_tab);
        uint32_t *yo = reinterpret_cast<uint32_t *>(xn + (size_t)row * D);
#pragma unroll
        for (int j = 0; j < NW; j++)
            yo[lane + 32 * j] = pack_low4(norm_b(x[j][0], w[j][0], nr), norm_b(x[j][1], w[j][1], nr),
                                          norm_b(x[j][2], w[j][2], nr), norm_b(x[j][3], w[j][3], nr));
    }
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
    const int lane = threadIdx.x & 31;
    const uint32_t *pw = reinterpret_cast<const uint32_t *>(post_w);
    const uint32_t *nw = reinterpret_cast<const uint32_t *>(next_w);
    int w[NW][4], w2[NW][4];
#pragma unroll
    for (int j = 0; j < NW; j++) {
        unpack4(__ldg(pw + lane + 32 * j), w[j]);
        unpack4(__ldg(nw + lane + 32 * j), w2[j]);
    }
    for (int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); row < M; row += row_warps()) {
        const uint32_t *ov = reinterpret_cast<const uint32_t *>(o + (size_t)row * D);
        RT *xr = x_res + (size_t)row * D;
        const uint32_t *er = MODE == kResFromEmbed ? reinterpret_cast<const uint32_t *>(embed + (size_t)tok_in[row] * D)
                                                   : nullptr;
        uint32_t x[NW];
        int4 rv[NW];
        int ss = 0;
#pragma unroll
        for (int j = 0; j < NW; j++) {   // every load of the row first
            x[j] = ov[lane + 32 * j];
            if (MODE == kResFromEmbed) {
                int ev[4];
                unpack4(__ldg(er + lane + 32 * j), ev);
                rv[j] = make_int4(ev[0], ev[1], ev[2], ev[3]);
            } else {
                rv[j] = load_res4(xr + 4 * (lane + 32 * j));
            }
        }
#pragma unroll
        for (int j = 0; j < NW; j++) ss = __dp4a((int)x[j], (int)x[j], ss);   // o is already clamped to +-127
        const NormRow n1 = norm_row(warp_sum(ss), D, inv_tab);
        int c[NW][4];
        int ss2 = 0;
#pragma unroll
        for (int j = 0; j < NW; j++) {
            int xo[4];
            unpack4(x[j], xo);
            int4 r = rv[j];
            r.x = (int)((uint32_t)r.x + (uint32_t)norm_b(xo[0], w[j][0], n1) - kM1Bits);
            r.y = (int)((uint32_t)r.y + (uint32_t)norm_b(xo[1], w[j][1], n1) - kM1Bits);
            r.z = (int)((uint32_t)r.z + (uint32_t)norm_b(xo[2], w[j][2], n1) - kM1Bits);
            r.w = (int)((uint32_t)r.w + (uint32_t)norm_b(xo[3], w[j][3], n1) - kM1Bits);
            if (MODE != kResNoStore) store_res4(xr + 4 * (lane + 32 * j), r);
            c[j][0] = clamp127(r.x);
            c[j][1] = clamp127(r.y);
            c[j][2] = clamp127(r.z);
            c[j][3] = clamp127(r.w);
#pragma unroll
            for (int b = 0; b < 4; b++) ss2 += c[j][b] * c[j][b];
        }
        const NormRow n2 = norm_row(warp_sum(ss2), D, inv_tab);
        uint32_t *yo = reinterpret_cast<uint32_t *>(xn + (size_t)row * D);
#pragma unroll
        for (int j = 0; j < NW; j++)
            yo[lane + 32 * j] = pack_low4(norm_b(c[j][0], w2[j][0], n2), norm_b(c[j][1], w2[j][1], n2),
                                          norm_b(c[j][2], w2[j][2], n2), norm_b(c[j][3], w2[j][3], n2));
    }
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
    dst[i] = (int8_t)rope_k_round(x * c - y * s);            // attention.rs:29-50
    dst[i + kHalfDim] = (int8_t)rope_k_round(x * s + y * c);
    reinterpret_cast<uint16_t *>(dst + 64)[i] = reinterpret_cast<const uint16_t *>(k + 64)[i];
}

// K rotated (attention.rs:29-50) and V of every row into its chunk's streaming
// layout (the tensor-core attention for chunks longer than its shared memory
// holds): chunk c at kv + (chunk_row0[c] + 32 c) * 128 bytes, its keys' K rows of
// 64 permuted dims (bytes [16t' + 4k + b] = dim 16k + 4t' + b) first, then V in
// 32-key tiles of 2 KB from npad * 64 on (npad = len rounded up to 32), byte
// (key, dim) at tile * 2048 + vt_byte(key % 32, dim) (lane-major, common.cuh) -- the
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
    kr[16 * ((i >> 2) & 3) + 4 * (i >> 4) + (i & 3)] = (int8_t)rope_k_round(x * cs - y * sn);
    kr[16 * ((i2 >> 2) & 3) + 4 * (i2 >> 4) + (i2 & 3)] = (int8_t)rope_k_round(x * sn + y * cs);
    int8_t *vt = base + (size_t)npad * 64 + (size_t)(p >> 5) * 2048;   // the V tile of key p (vt_byte)
    vt[vt_byte(p & 31, 2 * i)] = k[64 + 2 * i];
    vt[vt_byte(p & 31, 2 * i + 1)] = k[64 + 2 * i + 1];
}

// xn[r] = xn_tab[tok_in[r]], 16 bytes per thread (the table, V x d bytes, stays in L2)
__global__ void k_xn_gather(const uint32_t *__restrict__ tok_in, const int8_t *__restrict__ xn_tab, int M,
                            int chunks, int8_t *__restrict__ xn) {
    pdl_wait();
    pdl_trigger();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)M * chunks) return;
    const int row = (int)(i / chunks), c = (int)(i % chunks);
    const uint4 *src = reinterpret_cast<const uint4 *>(xn_tab) + (size_t)tok_in[row] * chunks + c;
    reinterpret_cast<uint4 *>(xn)[(size_t)row * chunks + c] = __ldg(src);
}

// ---- host launchers -------------------------------------------------------

void launch_rows(const uint32_t *tokens, const int *chunk_row0, const int *chunk_len,
                 const uint64_t *chunk_tok0, int n_chunks, int vocab, uint32_t *tok_in,
                 uint32_t *tok_out, int *pos, int *rowchunk, int *err, cudaStream_t st) {
    if (n_chunks == 0) return;
    k_rows<<<n_chunks, 256, 0, st>>>(tokens, chunk_row0, chunk_len, chunk_tok0, vocab, tok_in,
                                     tok_out, pos, rowchunk, err);
}

// row kernels: blocks of 8 warps, at most 8 blocks per SM resident at once (each warp
// then walks rows with a stride of the whole grid)
inline int row_blocks(int M) { return std::min((M + 7) / 8, 8 * sm_count()); }

template <typename RT, bool STORE>
void embed_norm_t(const uint32_t *tok_in, const int8_t *embed, const int8_t *norm_w, int M, int d, const uint16_t *inv_tab,
                  RT *x_res, int8_t *xn, cudaStream_t st) {
    const int blocks = row_blocks(M);
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
    const int blocks = row_blocks(M);
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

void launch_xn_gather(const uint32_t *tok_in, const int8_t *xn_tab, int M, int d, int8_t *xn, cudaStream_t st) {
    if (M == 0) return;
    const int chunks = d / 16;
    const long long n = (long long)M * chunks;
    launch_k(k_xn_gather, (unsigned)((n + 255) / 256), 256, 0, st, tok_in, xn_tab, M, chunks, xn);
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
