// coder.cu -- integer softmax -> CDF and the 32-bit arithmetic encoder.
//
// CDF: rust/src/softmax_cdf.rs:85-139.  For one row of int32 logits:
//   max and first argmax; e_i = exp_q16(l_i - max) (coef from the model file);
//   S = sum e_i; freq_i = 1 + floor(e_i * (T - V) / S); the argmax also takes
//   T - sum freq; cum = inclusive prefix sum.
// The encoder only needs the symbol's interval, so the compress path reduces
// the row to (sym_low, sym_high) = (cum[sym-1], cum[sym]) without storing cum.
// The division by the row-invariant S uses a 64-bit reciprocal with one
// correction step (exact, see udiv_by_inv).
//
// Encoder: rust/src/arith_coder.rs:8-136, one thread per chunk: interval update
// (80-98), E1/E2/E3 renormalisation with pending bits (101-119), MSB-first bit
// packing (51-62), finish = one '1' bit and a zero-padded last byte (122-130).
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

// one warp per row
__global__ void k_cdf_lohi(const int32_t *__restrict__ logits, int V, int ld,
                           const uint32_t *__restrict__ sym, const uint16_t *__restrict__ lut_g,
                           uint32_t coef, uint32_t total, int M, uint2 *__restrict__ lohi) {
    __shared__ uint16_t lut[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = lut_g[i];
    __syncthreads();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const int32_t *lg = logits + (size_t)row * ld;

    // max and its first index (argmax_deterministic, primitives.rs:278-295)
    int mx = INT32_MIN, am = 0x7fffffff;
    for (int i = lane; i < V; i += 32) {
        int v = lg[i];
        if (v > mx) { mx = v; am = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        int om = __shfl_xor_sync(0xffffffffu, mx, o);
        int oa = __shfl_xor_sync(0xffffffffu, am, o);
        if (om > mx || (om == mx && oa < am)) { mx = om; am = oa; }
    }
    // S = sum of exp weights (<= 65535 * V, fits 32 bits for V <= 65536)
    uint32_t S = 0;
    for (int i = lane; i < V; i += 32)
        S += exp_q16((int)((uint32_t)lg[i] - (uint32_t)mx), lut, coef);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);

    const unsigned long long R = (unsigned long long)(total - (uint32_t)V);
    const unsigned long long inv = 0xFFFFFFFFFFFFFFFFull / S;
    const uint32_t sy = sym[row];
    uint32_t f_all = 0, f_below = 0, f_sym = 0;
    for (int i = lane; i < V; i += 32) {
        uint32_t e = exp_q16((int)((uint32_t)lg[i] - (uint32_t)mx), lut, coef);
        uint32_t f = 1u + (uint32_t)udiv_by_inv((unsigned long long)e * R, S, inv);
        f_all += f;
        if ((uint32_t)i < sy) f_below += f;
        if ((uint32_t)i == sy) f_sym = f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        f_all += __shfl_xor_sync(0xffffffffu, f_all, o);
        f_below += __shfl_xor_sync(0xffffffffu, f_below, o);
        f_sym += __shfl_xor_sync(0xffffffffu, f_sym, o);
    }
    if (lane == 0) {
        uint32_t rem = total - f_all;   // goes to the argmax (softmax_cdf.rs:125-127)
        uint32_t lo = f_below + ((uint32_t)am < sy ? rem : 0u);
        uint32_t hi = lo + f_sym + ((uint32_t)am == sy ? rem : 0u);
        lohi[row] = make_uint2(lo, hi);
    }
}

// Register-resident version for V <= 128 * G (and so S < 2^26): the row is read
// once (lane l holds elements 128j + 4l + k), the weights e_i are kept packed,
// and the division by S uses freq_of.  The weight is read from lut4k,
// exp_q16 tabulated by t256 (entries >= 4096 are 1), with
// t256 = the high word of neg * (coef << 8) + 2^31, which needs coef < 2^24.
// Everything below the symbol is summed per block of 4 entries: the blocks
// 128j + 4l.. wholly below it add their block sums, and the one block that holds
// it (j = sym >> 7) is taken apart.  The first argmax lies below the symbol iff
// the maximum of the entries below it equals the row's maximum, and is the symbol
// iff it does not and the symbol's logit is the maximum.
// FULL: V == 128 * G, so no element is out of range.  EXP0: lut4k[0] == 65535 and
// |logit| < 2^30 (no wrap in logit - max), so a zero difference needs no special
// case.  One warp per row.
template <int G, bool FULL, bool EXP0>
__global__ void __launch_bounds__(256, 4) k_cdf_lohi_reg(const int32_t *__restrict__ logits, int V, int ld,
                                                      const uint32_t *__restrict__ sym,
                                                      const uint16_t *__restrict__ lut4k, uint32_t c8,
                                                      uint32_t total, int M, uint2 *__restrict__ lohi) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const int4 *src = reinterpret_cast<const int4 *>(logits + (size_t)row * ld);
    int x[G][4];
#pragma unroll
    for (int j = 0; j < G; j++) {
        int4 v = make_int4(INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN);
        if (FULL || 128 * j + 4 * lane < V) v = __ldcs(src + 32 * j + lane);   // read once: streaming
        x[j][0] = v.x; x[j][1] = v.y; x[j][2] = v.z; x[j][3] = v.w;
        if (!FULL) {   // a partly valid block
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (128 * j + 4 * lane + k >= V) x[j][k] = INT32_MIN;
        }
    }
    const int sy = (int)sym[row];
    const int J = sy >> 7;                  // block index of the symbol
    const int kk = (sy & 127) - 4 * lane;   // entries k < kk of this lane's block J lie below it
    // this lane's block J, the row max, and the max below the symbol
    int xJ[4] = {INT32_MIN, INT32_MIN, INT32_MIN, INT32_MIN};
    int mx = INT32_MIN, mb = INT32_MIN;
#pragma unroll
    for (int j = 0; j < G; j++) {
        const int bm = max(max(x[j][0], x[j][1]), max(x[j][2], x[j][3]));
        mx = max(mx, bm);
        if (j < J) mb = max(mb, bm);
        if (j == J) { xJ[0] = x[j][0]; xJ[1] = x[j][1]; xJ[2] = x[j][2]; xJ[3] = x[j][3]; }
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
        if (k < kk) mb = max(mb, xJ[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    }
    uint32_t ew[G][2];   // packed 16-bit weights
    uint32_t S = 0;
#pragma unroll
    for (int j = 0; j < G; j++) {
        uint32_t e[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int i = 128 * j + 4 * lane + k;
            const uint32_t neg = (uint32_t)mx - (uint32_t)x[j][k];
            const uint32_t t = min((uint32_t)(((unsigned long long)neg * c8 + 0x80000000ull) >> 32), 4096u);
            uint32_t w = __ldg(lut4k + t);
            if (!EXP0) w = neg == 0u ? 65535u : w;
            e[k] = (FULL || i < V) ? w : 0u;
            S += e[k];
        }
        ew[j][0] = e[0] | (e[1] << 16);
        ew[j][1] = e[2] | (e[3] << 16);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    const FreqDiv fd = make_freq_div(total - (uint32_t)V, S);
    uint32_t f_all = 0, f_below = 0, eJ[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < G; j++) {
        uint32_t fs = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t e = (ew[j][k >> 1] >> (16 * (k & 1))) & 0xFFFFu;
            uint32_t f = freq_of(e, fd);
            if (!FULL) f = 128 * j + 4 * lane + k < V ? f : 0u;
            fs += f;
        }
        f_all += fs;
        if (j < J) f_below += fs;
        if (j == J) { eJ[0] = ew[j][0]; eJ[1] = ew[j][1]; }
    }
    // block J entry by entry: those below the symbol, and the symbol itself
    uint32_t f_sym = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t f = freq_of((eJ[k >> 1] >> (16 * (k & 1))) & 0xFFFFu, fd);
        if (k < kk) f_below += f;
        if (k == kk) f_sym = f;
    }
    const int owner = (sy & 127) >> 2;
    f_sym = __shfl_sync(0xffffffffu, f_sym, owner);
    const int sk = sy & 3;
    const int xs = sk == 0 ? xJ[0] : sk == 1 ? xJ[1] : sk == 2 ? xJ[2] : xJ[3];
    const int x_sym = __shfl_sync(0xffffffffu, xs, owner);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        f_all += __shfl_xor_sync(0xffffffffu, f_all, o);
        f_below += __shfl_xor_sync(0xffffffffu, f_below, o);
    }
    if (lane == 0) {
        const uint32_t rem = total - f_all;   // goes to the first argmax (softmax_cdf.rs:125-127)
        const bool am_below = mb == mx, am_sym = !am_below && x_sym == mx;
        const uint32_t lo = f_below + (am_below ? rem : 0u);
        const uint32_t hi = lo + f_sym + (am_sym ? rem : 0u);
        lohi[row] = make_uint2(lo, hi);
    }
}

template <int G>
void cdf_reg(bool full, bool exp0, const int32_t *logits, int V, int ld, const uint32_t *sym, const uint16_t *lut4k,
             uint32_t c8, uint32_t total, int M, uint2 *lohi, unsigned grid, cudaStream_t st) {
    if (full && exp0) k_cdf_lohi_reg<G, true, true><<<grid, 256, 0, st>>>(logits, V, ld, sym, lut4k, c8, total, M, lohi);
    else if (full) k_cdf_lohi_reg<G, true, false><<<grid, 256, 0, st>>>(logits, V, ld, sym, lut4k, c8, total, M, lohi);
    else k_cdf_lohi_reg<G, false, false><<<grid, 256, 0, st>>>(logits, V, ld, sym, lut4k, c8, total, M, lohi);
}

// MSB-first bit output of one coder (arith_coder.rs:66-73, 122-131): bits gather in
// a 64-bit accumulator and leave as 4 bytes once 32 are there; bytes past the
// slot's capacity are counted but not written (the caller reports the overflow).
struct WordSink {
    uint8_t *out;
    uint32_t cap, len;
    unsigned long long acc;   // pending bits, right-aligned
    int n;                    // number of pending bits (< 32 between calls)
    bool overflow;

    __device__ __forceinline__ void put_byte(uint32_t v) {
        if (len < cap) out[len] = (uint8_t)v;
        else overflow = true;
        len++;
    }
    __device__ __forceinline__ void put_word() {   // the top 32 of n >= 32 pending bits
        n -= 32;
        const uint32_t w = (uint32_t)(acc >> n);
        if (len + 4 <= cap && (len & 3u) == 0u) {   // slots start 4-byte aligned
            *reinterpret_cast<uint32_t *>(out + len) = __byte_perm(w, 0u, 0x0123u);
            len += 4;
        } else {
#pragma unroll
            for (int q = 0; q < 4; q++) put_byte(w >> (24 - 8 * q));
        }
        acc &= (1ull << n) - 1ull;
    }
    __device__ __forceinline__ void push(uint32_t bits, int count) {   // count <= 32
        acc = (acc << count) | bits;
        n += count;
        if (n >= 32) put_word();
    }
    // finish (arith_coder.rs:122-131): a terminating '1', the partial byte padded with zeros
    __device__ __forceinline__ void finish() {
        push(1u, 1);
        const int pad = (8 - (n & 7)) & 7;
        acc <<= pad;
        n += pad;
        while (n >= 8) {
            n -= 8;
            put_byte((uint32_t)(acc >> n) & 0xFFu);
        }
    }
};

// One lane per chunk: the 32 chunks of a warp are encoded side by side, each lane
// walking its own chunk's (sym_low, sym_high) pairs, the next 8 loaded while the
// current 8 are coded.  The reference's renormalisation loop (arith_coder.rs:101-119) in
// closed form, one pass per symbol:
//  * E1/E2: the k = clz(low ^ high) leading bits that agree leave at once -- the
//    first, then the pending bits (its complement), then the other k - 1 -- and
//    low/high shift by k (low taking 0s, high 1s);
//  * E3: while bit 30 of low is 1 and bit 30 of high is 0 the reference repeats
//    the E3 step; j such steps keep bit 31, drop the j bits below it and add j
//    pending bits.  After an E3 step the top bits of low and high differ, so no
//    E1/E2 step follows within the symbol, and after the bulk E1/E2 step the E3
//    test is the only one left.
// Output leaves in 32-bit words; a pending run that does not fit one push (over
// 32 bits together with the symbol's agreeing bits) goes out in pieces.
constexpr int ENC_THREADS = 128;
constexpr int ENC_AHEAD = 8;   // interval pairs loaded ahead of the coding (an L2 round trip is several steps)

__global__ void __launch_bounds__(ENC_THREADS)
k_encode(const uint2 *__restrict__ lohi, const int *__restrict__ chunk_row0,
         const int *__restrict__ chunk_len, int n_chunks, uint32_t total,
         unsigned long long inv_total, uint8_t *__restrict__ slots,
         const uint64_t *__restrict__ slot_off, uint32_t *__restrict__ lens,
         int *__restrict__ err) {
    const int c = blockIdx.x * ENC_THREADS + threadIdx.x;
    if (c >= n_chunks) return;
    const int r0 = chunk_row0[c], n = chunk_len[c];
    WordSink bs;
    bs.out = slots + slot_off[c];
    bs.cap = (uint32_t)(slot_off[c + 1] - slot_off[c]);
    bs.len = 0; bs.acc = 0; bs.n = 0; bs.overflow = false;
    uint32_t low = 0, high = 0xFFFFFFFFu, pending = 0;
    const uint2 *src = lohi + r0;
    // the pairs in blocks of ENC_AHEAD: the next block is in flight while this one is coded
    uint2 cur[ENC_AHEAD];
#pragma unroll
    for (int k = 0; k < ENC_AHEAD; k++) cur[k] = k < n ? src[k] : make_uint2(0, 0);
    for (int i0 = 0; i0 < n; i0 += ENC_AHEAD) {
    uint2 nxt[ENC_AHEAD];
#pragma unroll
    for (int k = 0; k < ENC_AHEAD; k++) nxt[k] = i0 + ENC_AHEAD + k < n ? src[i0 + ENC_AHEAD + k] : make_uint2(0, 0);
#pragma unroll
    for (int k = 0; k < ENC_AHEAD; k++) {   // unrolled, so cur[k] stays in registers
        if (i0 + k >= n) break;
        const uint2 lh = cur[k];
        // interval update (arith_coder.rs:86-97); both ends stay inside [low, high]
        const unsigned long long range = (unsigned long long)high - low + 1ull;
        const uint32_t nh = low + (uint32_t)udiv_by_inv((unsigned long long)lh.y * range, total, inv_total) - 1u;
        low = low + (uint32_t)udiv_by_inv((unsigned long long)lh.x * range, total, inv_total);
        high = nh;
        const uint32_t x = low ^ high;
        const int k1 = (x & 0x80000000u) ? 0 : (x == 0u ? 32 : __clz(x));
        if (k1 > 0) {   // E1/E2 in bulk
            const uint32_t b = low >> 31;
            const uint32_t rest = k1 > 1 ? (uint32_t)(((unsigned long long)low << 1) >> (33 - k1)) & ((1u << (k1 - 1)) - 1u)
                                         : 0u;
            const uint32_t tot = pending + (uint32_t)k1;
            if (tot <= 32u) {
                const unsigned long long fill = b ? 0ull : ((1ull << pending) - 1ull);
                bs.push((uint32_t)(((unsigned long long)b << (tot - 1)) | (fill << (k1 - 1)) | rest), (int)tot);
            } else {   // a long pending run
                bs.push(b, 1);
                const uint32_t f = b ? 0u : 0xFFFFFFFFu;
                for (uint32_t run = pending; run > 0;) {
                    const int cnt = run > 31u ? 31 : (int)run;
                    bs.push(f & ((1u << cnt) - 1u), cnt);
                    run -= (uint32_t)cnt;
                }
                if (k1 > 1) bs.push(rest, k1 - 1);
            }
            pending = 0;
            low = (uint32_t)((unsigned long long)low << k1);
            high = (uint32_t)(((unsigned long long)high << k1) | ((1ull << k1) - 1ull));
        }
        if ((low & ~high & 0x40000000u) != 0u) {   // E3 in bulk
            const int j = min(__clz(~(low << 1)), __clz(high << 1));   // <= 31: bit 0 of ~(low << 1) is 1
            pending += (uint32_t)j;
            low = (low << j) & 0x7FFFFFFFu;
            high = (high << j) | 0x80000000u | ((1u << j) - 1u);
        }
    }
#pragma unroll
    for (int k = 0; k < ENC_AHEAD; k++) cur[k] = nxt[k];
    }
    bs.finish();
    lens[c] = bs.len;
    if (bs.overflow) atomicOr(err, kErrOverflow);
}

// Exclusive scan of the encoded chunk lengths into packed offsets (pack_off[0..n)),
// the total at pack_off[n]; one CTA of 1024 threads walking the chunks 1024 at a time.
__global__ void __launch_bounds__(1024) k_pack_offsets(const uint32_t *__restrict__ lens, int n,
                                                       uint64_t *__restrict__ pack_off) {
    __shared__ uint64_t wsum[32];
    __shared__ uint64_t carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int b = 0; b < n; b += 1024) {
        const int i = b + (int)threadIdx.x;
        const uint64_t v = i < n ? lens[i] : 0;
        uint64_t x = v;   // inclusive scan in the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {   // scan of the warp totals
            uint64_t w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            wsum[lane] = w;
        }
        __syncthreads();
        const uint64_t before = carry + (warp ? wsum[warp - 1] : 0);
        if (i < n) pack_off[i] = before + x - v;
        __syncthreads();
        if (threadIdx.x == 0) carry += wsum[31];
        __syncthreads();
    }
    if (threadIdx.x == 0) pack_off[n] = carry;
}

// one CTA per chunk: slot bytes -> packed position
__global__ void k_pack(const uint8_t *__restrict__ slots, const uint64_t *__restrict__ slot_off,
                       const uint32_t *__restrict__ lens, const uint64_t *__restrict__ pack_off,
                       uint8_t *__restrict__ packed) {
    const int c = blockIdx.x;
    const uint8_t *src = slots + slot_off[c];
    uint8_t *dst = packed + pack_off[c];
    const uint32_t n = lens[c];
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

void launch_cdf_lohi(const int32_t *logits, int V, int ld, const uint32_t *sym, const uint16_t *lut,
                     const uint16_t *lut4k, bool exp0, uint32_t coef, uint32_t total, int M, uint2 *lohi,
                     cudaStream_t st) {
    if (M == 0) return;
    const unsigned grid = (unsigned)((M + 7) / 8);
    // 16-byte row loads need ld % 4 == 0; the weight bound needs V <= 1024; the table index coef < 2^24
    if (ld % 4 == 0 && V <= 1024 && coef < (1u << 24)) {
        const bool full = V % 128 == 0;
        const uint32_t c8 = coef << 8;
        switch ((V + 127) / 128) {
            case 8: cdf_reg<8>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 7: cdf_reg<7>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 6: cdf_reg<6>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 5: cdf_reg<5>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 4: cdf_reg<4>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 3: cdf_reg<3>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            case 2: cdf_reg<2>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
            default: cdf_reg<1>(full, exp0, logits, V, ld, sym, lut4k, c8, total, M, lohi, grid, st); return;
        }
    }
    k_cdf_lohi<<<grid, 256, 0, st>>>(logits, V, ld, sym, lut, coef, total, M, lohi);
}

void launch_encode(const uint2 *lohi, const int *chunk_row0, const int *chunk_len, int n_chunks,
                   uint32_t total, uint8_t *slots, const uint64_t *slot_off, uint32_t *lens,
                   int *err, cudaStream_t st) {
    if (n_chunks == 0) return;
    unsigned long long inv = 0xFFFFFFFFFFFFFFFFull / total;
    k_encode<<<(n_chunks + ENC_THREADS - 1) / ENC_THREADS, ENC_THREADS, 0, st>>>(
        lohi, chunk_row0, chunk_len, n_chunks, total, inv, slots, slot_off, lens, err);
}

void launch_pack_offsets(const uint32_t *lens, int n_chunks, uint64_t *pack_off, cudaStream_t st) {
    k_pack_offsets<<<1, 1024, 0, st>>>(lens, n_chunks, pack_off);
}

void launch_pack(const uint8_t *slots, const uint64_t *slot_off, const uint32_t *lens,
                 const uint64_t *pack_off, int n_chunks, uint8_t *packed, cudaStream_t st) {
    if (n_chunks == 0) return;
    k_pack<<<n_chunks, 128, 0, st>>>(slots, slot_off, lens, pack_off, packed);
}

}  // namespace czg
