// decode.cu -- batched decompression: many chunks decode in lockstep, one token
// per chunk per step (the loop of rust/src/main.rs:377-396 for every chunk).
//
// Per step the model kernels run on the M active streams (rows), the new K/V
// row is appended to each stream's int8 cache, and k_cdf_decode turns each
// stream's logits into its CDF (rust/src/softmax_cdf.rs:85-139) and runs one
// ArithDecoder::decode_symbol (rust/src/arith_coder.rs:195-264) on it, one warp
// per stream; the decoded symbol is the next step's input token.
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

// bit `bit` of the chunk, MSB first; reads past the end give 0 (arith_coder.rs:176-190)
__device__ __forceinline__ uint32_t read_bit(const uint8_t *data, uint64_t len, uint64_t bit) {
    const uint64_t byte = bit >> 3;
    if (byte >= len) return 0u;
    return (uint32_t)(data[byte] >> (7 - (bit & 7))) & 1u;
}

// Byte `lane` (< 9) of the chunk from the byte holding bit `bit` on, 0 past the end;
// window() assembles the warp's nine bytes into the 64 bits from `bit` on, MSB first.
__device__ __forceinline__ uint32_t window_byte(const uint8_t *data, uint64_t len, uint64_t bit, int lane) {
    const uint64_t byte = (bit >> 3) + (uint64_t)lane;
    return (lane < 9 && byte < len) ? (uint32_t)data[byte] : 0u;
}
__device__ __forceinline__ unsigned long long window(uint32_t b, uint64_t bit, int lane) {
    const uint32_t hi = __reduce_or_sync(0xffffffffu, lane < 4 ? b << (24 - 8 * lane) : 0u);
    const uint32_t lo = __reduce_or_sync(0xffffffffu, lane >= 4 && lane < 8 ? b << (56 - 8 * lane) : 0u);
    const uint32_t b8 = __shfl_sync(0xffffffffu, b, 8);
    const unsigned long long w = ((unsigned long long)hi << 32) | lo;
    const int off = (int)(bit & 7);
    return off ? (w << off) | (b8 >> (8 - off)) : w;
}

// ArithDecoder::decode_symbol after the search (arith_coder.rs:244-264): narrow to
// [lo, hi) of total, then renormalise in closed form.  The loop shifts while the top
// bits of low and high agree (n1 = clz(low ^ high) times, 32 when equal), and only
// then takes the E3 steps, while bit 30 is set in low and clear in high: an E3 step
// leaves the top bits different, so no E1/E2 step follows one.  Over k steps
//   E1/E2: low << k, (high << k) | (2^k - 1), (code << k) | next k bits;
//   E3:    (low << k) ^ HALF, (high << k) | HALF | (2^k - 1),
//          (code & HALF) | ((code << k) & (HALF - 1)) | next k bits,
// with n3 = the run of set bits of low & ~high from bit 30 down.  n1 + n3 <= 63, so
// the 64-bit window `win` holds every bit read.
__device__ __forceinline__ void dec_narrow(DecState &s, uint32_t lo, uint32_t hi, uint32_t total,
                                           unsigned long long inv_total, unsigned long long win) {
    const unsigned long long range = (unsigned long long)s.high - s.low + 1;
    uint32_t high = (uint32_t)(s.low + udiv_by_inv((unsigned long long)hi * range, total, inv_total) - 1);
    uint32_t low = (uint32_t)(s.low + udiv_by_inv((unsigned long long)lo * range, total, inv_total));
    uint32_t code = s.code;
    const int n1 = __clz((int)(low ^ high));
    if (n1 > 0) {
        low = (uint32_t)((unsigned long long)low << n1);
        high = (uint32_t)(((unsigned long long)high << n1) | ((1ull << n1) - 1ull));
        code = (uint32_t)(((unsigned long long)code << n1) | (win >> (64 - n1)));
        win <<= n1;
    }
    const int n3 = __clz((int)~((low & ~high) << 1));
    if (n3 > 0) {
        low = (low << n3) ^ 0x80000000u;
        high = (high << n3) | 0x80000000u | ((1u << n3) - 1u);
        code = (code & 0x80000000u) | ((code << n3) & 0x7FFFFFFFu) | (uint32_t)(win >> (64 - n3));
    }
    s.low = low;
    s.high = high;
    s.code = code;
    s.bit += (uint64_t)(n1 + n3);
}

// The next step's first pre-norm output of a stream decoded to `sym`: row sym of the
// normalised embedding table (the first norm of a row depends on its token alone).
__device__ __forceinline__ void copy_xn_row(const int8_t *__restrict__ xn_tab, int8_t *__restrict__ xn, int d,
                                            uint32_t sym, int r, int lane) {
    const uint32_t *src = reinterpret_cast<const uint32_t *>(xn_tab + (size_t)sym * d);
    uint32_t *dst = reinterpret_cast<uint32_t *>(xn + (size_t)r * d);
    for (int j = lane; j < d / 4; j += 32) dst[j] = __ldg(src + j);
}

// ArithDecoder::new: code = the first 32 bits (arith_coder.rs:153-174)
__global__ void k_dec_init(const uint8_t *__restrict__ data, const uint64_t *__restrict__ data_off,
                           const uint64_t *__restrict__ data_len, int M, DecState *__restrict__ st,
                           uint32_t *__restrict__ tok_in) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= M) return;
    const uint8_t *d = data + data_off[r];
    const uint64_t len = data_len[r];
    uint32_t code = 0;
    for (int i = 0; i < 32; i++) code = (code << 1) | read_bit(d, len, (uint64_t)i);
    DecState s;
    s.low = 0;
    s.high = 0xFFFFFFFFu;
    s.code = code;
    s.pad = 0;
    s.bit = 32;
    st[r] = s;
    tok_in[r] = kBos;
}

// rows of the batch at position pos: K rotated (attention.rs:29-50) and V into the cache.
// split == false: the row is [k_rot 64 | v 64] at pos * 128.  split == true (the
// tensor-core decode attention): K at pos * 64 with its dims permuted as
// bytes [16t' + 4k + b] = dim 16k + 4t' + b, and V from len * 64 on in 32-key tiles
// of 2 KB, byte (key, dim) at tile * 2048 + vt_byte(key % 32, dim) (lane-major,
// common.cuh), where len = cache_ld / 128.
__global__ void k_kv_append(const int8_t *__restrict__ qkv, int ldq, int d, int pos,
                            const int16_t *__restrict__ rope_cos, const int16_t *__restrict__ rope_sin,
                            int M, int8_t *__restrict__ kvc, size_t cache_ld, bool split) {
    pdl_wait();
    pdl_trigger();
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const int r = gid >> 5, i = gid & 31;
    if (r >= M) return;
    const int8_t *k = qkv + (size_t)r * ldq + d;
    const int x = k[i], y = k[i + kHalfDim];
    const int c = rope_cos[pos * kHalfDim + i], s = rope_sin[pos * kHalfDim + i];
    const int8_t kx = (int8_t)rope_k_round(x * c - y * s);
    const int8_t ky = (int8_t)rope_k_round(x * s + y * c);
    int8_t *base = kvc + (size_t)r * cache_ld;
    if (!split) {
        int8_t *dst = base + (size_t)pos * 128;
        dst[i] = kx;
        dst[i + kHalfDim] = ky;
        reinterpret_cast<uint16_t *>(dst + 64)[i] = reinterpret_cast<const uint16_t *>(k + 64)[i];
    } else {
        const size_t len = cache_ld / 128;
        int8_t *kr = base + (size_t)pos * 64;
        const int i2 = i + kHalfDim;
        kr[16 * ((i >> 2) & 3) + 4 * (i >> 4) + (i & 3)] = kx;
        kr[16 * ((i2 >> 2) & 3) + 4 * (i2 >> 4) + (i2 & 3)] = ky;
        int8_t *vt = base + len * 64 + (size_t)(pos >> 5) * 2048;   // the V tile of key pos
        vt[vt_byte(pos & 31, 2 * i)] = k[64 + 2 * i];
        vt[vt_byte(pos & 31, 2 * i + 1)] = k[64 + 2 * i + 1];
    }
}

// One warp per stream: CDF of the logits row, then one decode_symbol.
// Lane l owns vocabulary entries [l*E, min((l+1)*E, V)), E = ceil(V / 32).
__global__ void k_cdf_decode(const int32_t *__restrict__ logits, int V, int ld, const uint16_t *__restrict__ lut_g,
                             uint32_t coef, uint32_t total, unsigned long long inv_total, int M,
                             DecState *__restrict__ st, const uint8_t *__restrict__ data,
                             const uint64_t *__restrict__ data_off, const uint64_t *__restrict__ data_len,
                             const uint64_t *__restrict__ tok_off, int step, uint32_t *__restrict__ out_tok,
                             uint32_t *__restrict__ tok_in, const int8_t *__restrict__ xn_tab,
                             int8_t *__restrict__ xn, int d) {
    __shared__ uint16_t lut[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = lut_g[i];   // model constant
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= M) return;
    const int32_t *lg = logits + (size_t)r * ld;
    const int E = (V + 31) >> 5;
    const int i0 = min(V, lane * E), i1 = min(V, i0 + E);

    // max and first argmax (primitives.rs:278-295)
    int mx = INT32_MIN, am = 0x7fffffff;
    for (int i = i0; i < i1; i++) {
        const int v = lg[i];
        if (v > mx) { mx = v; am = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const int om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oa = __shfl_xor_sync(0xffffffffu, am, o);
        if (om > mx || (om == mx && oa < am)) { mx = om; am = oa; }
    }
    uint32_t S = 0;
    for (int i = i0; i < i1; i++) S += exp_q16((int)((uint32_t)lg[i] - (uint32_t)mx), lut, coef);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    const unsigned long long R = (unsigned long long)(total - (uint32_t)V);
    const unsigned long long invS = 0xFFFFFFFFFFFFFFFFull / S;
    uint32_t F = 0;
    for (int i = i0; i < i1; i++) {
        const uint32_t e = exp_q16((int)((uint32_t)lg[i] - (uint32_t)mx), lut, coef);
        F += 1u + (uint32_t)udiv_by_inv((unsigned long long)e * R, S, invS);
    }
    uint32_t all = F;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) all += __shfl_xor_sync(0xffffffffu, all, o);
    const uint32_t rem = total - all;   // to the argmax (softmax_cdf.rs:125-127)
    if (am >= i0 && am < i1) F += rem;
    uint32_t inc = F;   // inclusive scan of lane totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
    }
    const uint32_t base = inc - F;

    DecState s = st[r];
    const unsigned long long range = (unsigned long long)s.high - s.low + 1;
    // value = ((code - low + 1) * T - 1) / range  (arith_coder.rs:195-200)
    const unsigned long long value = (((unsigned long long)s.code - s.low + 1) * total - 1) / range;
    // bisect on the value truncated to 32 bits (arith_coder.rs:203, 225-241): smallest i
    // with v32 < cum[i], else the last symbol
    const uint32_t v32 = (uint32_t)value;
    const bool mine = i0 < i1 && v32 >= base && v32 < base + F;
    const uint32_t bal = __ballot_sync(0xffffffffu, mine);
    const bool past_end = bal == 0;
    const unsigned owner = past_end ? (unsigned)((V - 1) / E) : (unsigned)(__ffs(bal) - 1);
    uint32_t sym = 0, lo = 0, hi = 0;
    if (lane == (int)owner) {
        uint32_t cum = base;
        for (int i = i0; i < i1; i++) {
            const uint32_t e = exp_q16((int)((uint32_t)lg[i] - (uint32_t)mx), lut, coef);
            uint32_t f = 1u + (uint32_t)udiv_by_inv((unsigned long long)e * R, S, invS);
            if (i == am) f += rem;
            if ((!past_end && v32 < cum + f) || (past_end && i == V - 1)) {
                sym = (uint32_t)i;
                lo = cum;
                hi = cum + f;
                break;
            }
            cum += f;
        }
    }
    sym = __shfl_sync(0xffffffffu, sym, owner);
    lo = __shfl_sync(0xffffffffu, lo, owner);
    hi = __shfl_sync(0xffffffffu, hi, owner);
    if (lane == 0) {
        const unsigned long long HALF = 1ull << 31, QUARTER = 1ull << 30, MASK = 0xFFFFFFFFull;
        unsigned long long low = s.low, high = s.high, code = s.code;
        uint64_t bit = s.bit;
        const uint8_t *d = data + data_off[r];
        const uint64_t len = data_len[r];
        high = low + udiv_by_inv((unsigned long long)hi * range, total, inv_total) - 1;
        low = low + udiv_by_inv((unsigned long long)lo * range, total, inv_total);
        for (;;) {   // arith_coder.rs:244-264
            if (((low ^ high) & HALF) == 0) {
                low = (low << 1) & MASK;
                high = ((high << 1) & MASK) | 1ull;
                code = ((code << 1) & MASK) | read_bit(d, len, bit++);
            } else if ((low & ~high & QUARTER) != 0) {
                low = ((low << 1) ^ HALF) & MASK;
                high = (((high ^ HALF) << 1) | HALF | 1ull) & MASK;
                code = (code & HALF) | ((code << 1) & (MASK >> 1)) | read_bit(d, len, bit++);
            } else {
                break;
            }
        }
        s.low = (uint32_t)low;
        s.high = (uint32_t)high;
        s.code = (uint32_t)code;
        s.bit = bit;
        st[r] = s;
        out_tok[tok_off[r] + step] = sym;
        tok_in[r] = sym;
    }
    if (xn != nullptr) copy_xn_row(xn_tab, xn, d, sym, r, lane);
}

// Register-resident version for V == 32 * E (E in {8, 16, 32}): lane l holds the
// E consecutive logits [l*E, (l+1)*E) in registers (each warp copies its next
// stream's row, coder state and offsets into shared memory while it decodes the
// current one), the weights come from the
// t256-indexed table lut4k (needs coef < 2^24), the division by S uses
// freq_of.  The interval search is done by the whole warp: the owner
// lane's weights go through shared memory, one element per lane, and an
// inclusive scan gives the cumulative frequencies.  Persistent (CDF_BLOCKS_PER_SM
// blocks per SM, warp w takes streams w, w + W, ...), with the table in shared
// memory: its 32 x E random lookups per stream are gathers that the L1 path
// serves one cache line at a time, shared memory one bank conflict at a time.
constexpr int CDF_LUT_WORDS = 4104 / 2;   // lut4k: t256 0..4096, padded
constexpr int CDF_BLOCKS_PER_SM = 4;

// KEY: every logit is below 2^26 in magnitude (d * 127 * 128 < 2^26), so
// logit * 32 + (31 - k) orders the lane's entries by value, then by first index, in
// one int32 and the lane's max with its first index is a three-input max tree.
template <int E, bool EXP0, bool KEY>
__global__ void __launch_bounds__(256, CDF_BLOCKS_PER_SM) k_cdf_decode_reg(
    const int32_t *__restrict__ logits, int ld, const uint16_t *__restrict__ lut4k_g, uint32_t c8, uint32_t total,
    unsigned long long inv_total, int M, DecState *__restrict__ st, const uint8_t *__restrict__ data,
    const uint64_t *__restrict__ data_off, const uint64_t *__restrict__ data_len, const uint64_t *__restrict__ tok_off,
    int step, uint32_t *__restrict__ out_tok, uint32_t *__restrict__ tok_in, const int8_t *__restrict__ xn_tab,
    int8_t *__restrict__ xn, int d) {
    constexpr int V = 32 * E;
    __shared__ uint32_t ebuf[8][E / 2];
    __shared__ uint32_t lut_w[CDF_LUT_WORDS];
    __shared__ __align__(16) int4 rowbuf[8][V / 4];   // per warp: its next stream's logits
    // and that stream's coder state (3 words of 8 bytes), chunk offset, length and token offset
    __shared__ __align__(16) unsigned long long mbuf[8][8];
    for (int i = threadIdx.x; i < CDF_LUT_WORDS; i += blockDim.x)   // model constant: before the wait
        lut_w[i] = __ldg(reinterpret_cast<const uint32_t *>(lut4k_g) + i);
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    const uint16_t *lut4k = reinterpret_cast<const uint16_t *>(lut_w);
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int stride = gridDim.x * 8;
    // the logits row of stream r into rowbuf with cp.async, 16-byte chunk c at c ^ ((c >> 3) & 7):
    // lane l later reads its chunks l * E / 4 + k, and the eight lanes of each phase of a
    // 16-byte shared load then fall on eight different bank groups
    auto fetch_row = [&](int r) {
        if (r < M) {
            const int4 *src = reinterpret_cast<const int4 *>(logits + (size_t)r * ld);
#pragma unroll
            for (int c = lane; c < V / 4; c += 32)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                                 (uint32_t)__cvta_generic_to_shared(&rowbuf[wib][c ^ ((c >> 3) & 7)])),
                             "l"(src + c)
                             : "memory");
            if (lane < 6) {
                const void *m8 = lane < 3 ? static_cast<const void *>(reinterpret_cast<const uint64_t *>(st + r) + lane)
                                 : lane == 3 ? static_cast<const void *>(data_off + r)
                                 : lane == 4 ? static_cast<const void *>(data_len + r)
                                             : static_cast<const void *>(tok_off + r);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(
                                 (uint32_t)__cvta_generic_to_shared(&mbuf[wib][lane])),
                             "l"(m8)
                             : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch_row(blockIdx.x * 8 + wib);
    for (int r = blockIdx.x * 8 + wib; r < M; r += stride) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    int x[E];
#pragma unroll
    for (int k = 0; k < E / 4; k++) {
        const int c = lane * (E / 4) + k;
        const int4 v = rowbuf[wib][c ^ ((c >> 3) & 7)];
        x[4 * k] = v.x; x[4 * k + 1] = v.y; x[4 * k + 2] = v.z; x[4 * k + 3] = v.w;
    }
    DecState s = *reinterpret_cast<const DecState *>(&mbuf[wib][0]);
    const unsigned long long doff = mbuf[wib][3], dlen = mbuf[wib][4], toff = mbuf[wib][5];
    __syncwarp();   // the buffers take the warp's next stream while this one is decoded
    fetch_row(r + stride);
    // the next 9 bytes of the chunk, loaded while the CDF is built
    const uint32_t wb = window_byte(data + doff, dlen, s.bit, lane);
    // max and first argmax (primitives.rs:278-295)
    int mx = INT32_MIN, am = 0x7fffffff;
    if constexpr (KEY) {
        int key = INT32_MIN;
#pragma unroll
        for (int k = 0; k < E; k += 2) key = __vimax3_s32(key, x[k] * 32 + (31 - k), x[k + 1] * 32 + (30 - k));
        const int lmx = key >> 5;
        mx = lmx;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int first = __ffs(__ballot_sync(0xffffffffu, lmx == mx)) - 1;   // lowest lane holding the max
        am = first * E + 31 - (__shfl_sync(0xffffffffu, key, first) & 31);
    } else {
#pragma unroll
        for (int k = 0; k < E; k++)
            if (x[k] > mx) { mx = x[k]; am = lane * E + k; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int om = __shfl_xor_sync(0xffffffffu, mx, o);
            const int oa = __shfl_xor_sync(0xffffffffu, am, o);
            if (om > mx || (om == mx && oa < am)) { mx = om; am = oa; }
        }
    }
    uint32_t ew[E / 2];
    uint32_t S = 0;
#pragma unroll
    for (int k = 0; k < E; k++) {
        const int dlt = (int)((uint32_t)x[k] - (uint32_t)mx);
        const uint32_t neg = 0u - (uint32_t)dlt;
        const uint32_t t = min((uint32_t)(((unsigned long long)neg * c8 + 0x80000000ull) >> 32), 4096u);
        const uint32_t w = (EXP0 || dlt < 0) ? (uint32_t)lut4k[t] : 65535u;   // EXP0: lut4k[0] == 65535
        S += w;
        if (k & 1) ew[k >> 1] |= w << 16;
        else ew[k >> 1] = w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    const FreqDiv fd = make_freq_div(total - (uint32_t)V, S);
    uint32_t F = 0;
#pragma unroll
    for (int k = 0; k < E; k++) F += freq_of((ew[k >> 1] >> (16 * (k & 1))) & 0xFFFFu, fd);
    uint32_t all = F;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) all += __shfl_xor_sync(0xffffffffu, all, o);
    const uint32_t rem = total - all;   // to the argmax (softmax_cdf.rs:125-127)
    if (am / E == lane) F += rem;
    uint32_t inc = F;   // inclusive scan of lane totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
    }
    const uint32_t base = inc - F;

    const unsigned long long range = (unsigned long long)s.high - s.low + 1;
    // value = ((code - low + 1) * T - 1) / range  (arith_coder.rs:195-200), and the search
    // takes the smallest i with v32 < cum[i], else the last symbol (arith_coder.rs:203,
    // 225-241), v32 = value mod 2^32.  With code >= low (every stream the encoder wrote),
    // c = code - low + 1 <= range, so value < T < 2^30 is v32 and, for X < 2^31,
    // v32 < X  <=>  c * T - 1 < X * range  (both sides < 2^63): no division.  A corrupt
    // state (code < low) wraps c and takes the division.
    const unsigned long long cN = (unsigned long long)s.code - s.low + 1;
    const bool direct = cN <= range;   // the same for the whole warp
    const unsigned long long num = cN * total - 1;
    const uint32_t v32 = direct ? 0u : (uint32_t)(num / range);
    auto below = [&](uint32_t X) { return direct ? num < (unsigned long long)X * range : v32 < X; };
    const uint32_t bal = __ballot_sync(0xffffffffu, !below(base) && below(base + F));
    const bool past_end = bal == 0;
    const int owner = past_end ? 31 : __ffs(bal) - 1;
    if (lane == owner) {
#pragma unroll
        for (int k = 0; k < E / 2; k++) ebuf[wib][k] = ew[k];
    }
    const uint32_t obase = __shfl_sync(0xffffffffu, base, owner);
    __syncwarp();
    // lane j < E takes element owner*E + j
    uint32_t f = 0;
    const int idx = owner * E + lane;
    if (lane < E) {
        const uint32_t e = (ebuf[wib][lane >> 1] >> (16 * (lane & 1))) & 0xFFFFu;
        f = freq_of(e, fd) + (idx == am ? rem : 0u);
    }
    uint32_t cum = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, cum, o);
        if (lane >= o) cum += u;
    }
    cum += obase;
    const uint32_t hit = __ballot_sync(0xffffffffu, lane < E && below(cum));
    const int sl = past_end ? E - 1 : __ffs(hit) - 1;   // hit != 0 unless past the end
    const uint32_t hi = __shfl_sync(0xffffffffu, cum, sl);
    const uint32_t lo = hi - __shfl_sync(0xffffffffu, f, sl);
    const unsigned long long win = window(wb, s.bit, lane);
    const uint32_t sym = (uint32_t)(owner * E + sl);
    if (lane == 0) {
        dec_narrow(s, lo, hi, total, inv_total, win);
        st[r] = s;
        out_tok[toff + step] = sym;
        tok_in[r] = sym;
    }
    if (xn != nullptr) copy_xn_row(xn_tab, xn, d, sym, r, lane);
    __syncwarp();   // ebuf is rewritten for the warp's next stream
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

}  // namespace

void launch_dec_init(const uint8_t *data, const uint64_t *data_off, const uint64_t *data_len, int M,
                     DecState *st, uint32_t *tok_in, cudaStream_t stream) {
    if (M == 0) return;
    k_dec_init<<<(M + 127) / 128, 128, 0, stream>>>(data, data_off, data_len, M, st, tok_in);
}

void launch_kv_append(const int8_t *qkv, int ldq, int d, int pos, const int16_t *rope_cos,
                      const int16_t *rope_sin, int M, int8_t *kvc, size_t cache_ld, bool split, cudaStream_t stream) {
    if (M == 0) return;
    const long long threads = (long long)M * 32;
    launch_k(k_kv_append, (unsigned)((threads + 255) / 256), 256, 0, stream, qkv, ldq, d, pos, rope_cos, rope_sin, M,
             kvc, cache_ld, split);
}

void launch_cdf_decode(const int32_t *logits, int V, int ld, const uint16_t *lut, const uint16_t *lut4k, bool exp0,
                       uint32_t coef, uint32_t total, int M, DecState *st, const uint8_t *data,
                       const uint64_t *data_off, const uint64_t *data_len, const uint64_t *tok_off, int step,
                       uint32_t *out_tok, uint32_t *tok_in, const int8_t *xn_tab, int8_t *xn, int d,
                       cudaStream_t stream) {
    if (M == 0) return;
    const unsigned long long inv = 0xFFFFFFFFFFFFFFFFull / total;
    const unsigned grid = (unsigned)((M + 7) / 8);
    if (coef < (1u << 24) && ld % 4 == 0 && (V == 1024 || V == 512 || V == 256)) {
        const unsigned pgrid = std::min<unsigned>(grid, (unsigned)(CDF_BLOCKS_PER_SM * sm_count()));
        const uint32_t c8 = coef << 8;
        const bool key = (long long)d * 16256 < (1ll << 26);   // |logit| <= d * 127 * 128
#define CZG_CDF_DEC1(EE, X0, KY)                                                                                  \
    launch_k(k_cdf_decode_reg<EE, X0, KY>, pgrid, 256, 0, stream, logits, ld, lut4k, c8, total, inv, M, st, data, \
             data_off, data_len, tok_off, step, out_tok, tok_in, xn_tab, xn, d)
#define CZG_CDF_DEC(EE)                                                                                          \
    do {                                                                                                          \
        if (exp0 && key) CZG_CDF_DEC1(EE, true, true);                                                           \
        else if (exp0) CZG_CDF_DEC1(EE, true, false);                                                            \
        else if (key) CZG_CDF_DEC1(EE, false, true);                                                             \
        else CZG_CDF_DEC1(EE, false, false);                                                                     \
    } while (0)
        if (V == 1024) CZG_CDF_DEC(32);
        else if (V == 512) CZG_CDF_DEC(16);
        else CZG_CDF_DEC(8);
#undef CZG_CDF_DEC
#undef CZG_CDF_DEC1
        return;
    }
    launch_k(k_cdf_decode, grid, 256, 0, stream, logits, V, ld, lut, coef, total, inv, M, st, data, data_off, data_len,
             tok_off, step, out_tok, tok_in, xn_tab, xn, d);
}

}  // namespace czg
