// attention_mma.cu -- exact causal integer attention on the tensor cores.
//
// Same result as rust/src/attention.rs:162-289 run for positions 0..n-1 of a
// chunk (see attention.cu for the scalar form).  One CTA per chunk stages the
// chunk's K (RoPE applied) and V in shared memory; its 16 warps take tasks of
// 8 query rows of one head, longest rows first, and walk their keys in tiles
// of 32.
//
// QK^T: mma.sync m16n8k32 s8*s8 -> s32 gives the exact int32 dot products (the
// task's 8 rows are A rows 0..7; rows 8..15 are zero).  The key order inside a
// tile is permuted so that thread t of a quad holds the 8 consecutive keys
// 8t..8t+7 of its row g, which are also exactly the keys of its P fragment.
//
// Online softmax: per row, scores -> prefix max in key order (thread-local run
// + one quad scan) -> records (keys beating everything before them) -> weights
// w = exp(score - max so far) and rescale factors e = exp(old max - score).
//
// P*V is computed transposed, O^T = V^T * P^T (64 dims as the MMA's M, the 8
// rows as its N): the P^T fragment a thread supplies is its own row's weights.
// The 16-bit weights are split into a high and a low byte and multiplied with
// V (s8) as two s8*u8 MMAs into separate accumulators Hi, Lo; each is exactly
// sum(byte * v) and never overflows (|sum| <= 255*127*4096), so
// vacc = 256*Hi + Lo (mod 2^32) equals the reference's wrapping i32 sum; an
// all-ones A operand gives the weight sums.
// A tile whose rows contain records is replayed in passes: pass q adds the keys
// of segment q (segment = run of keys between records).  Before pass q every
// row with a q-th record in the tile folds its state exactly as the reference
// rescales at that key: Lo = R(256*Hi + Lo, e), Hi = 0, so the folded value
// lives on in the Lo accumulator (the MMA's s32 accumulation wraps modulo 2^32
// like the reference's i32 sum), and s = ((s + seg_sum) * e + 2^15) >> 16 (kept
// as an offset to the running weight sums).  The state stays in registers in
// the accumulator layout (row 2t+e of thread (g, t)), each row folded by the 8
// threads that hold it.  A record whose previous maximum is still INT32_MIN
// rescales nothing (attention.rs:248-250) and is no segment boundary.
// Record bookkeeping per tile: each thread's 8-bit record mask, the row's 32-bit
// mask (one bit per key), the records' (previous max - score) stored by key in
// shared memory; a folding thread walks its rows' masks lowest bit first.
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int AM_THREADS = 512;
constexpr int AM_WARPS = AM_THREADS / 32;
constexpr int AM_MAX_KEYS = 1024;
constexpr int AM_ROWS = 8;   // query rows per warp task
constexpr int AM_TASK_BATCH = 4;   // streamed kernel: consecutive tasks per counter increment
constexpr int AM_LUT = 4104;   // exp table entries (t256 0..4096, padded)
// per warp: record differences by key [8][32], output staging [8][64]
constexpr int AM_WARP_SMEM = AM_ROWS * 32 * 4 + AM_ROWS * 64;

__device__ __forceinline__ void mma_s8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8u8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// c = A * B from a zero accumulator (the previous contents of c are not read)
__device__ __forceinline__ void mma_s8u8_z(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// exp_q16 with the attention coefficient via a table indexed by min(t256, 4096)
// (entry 4096 is 1, the value of every t256 >= 4096, whatever the exp2 LUT holds);
// the kernels keep the table (8 KB) in shared memory.
// t256 = floor((neg * coef + 2^23) / 2^24) = the high word of neg * (coef << 8) + 2^31.
__device__ __forceinline__ uint32_t exp_attn(int diff, const uint16_t *lut4k, uint32_t c8) {
    const uint32_t neg = 0u - (uint32_t)diff;
    const uint32_t t = min((uint32_t)(((unsigned long long)neg * c8 + 0x80000000ull) >> 32), 4096u);
    const uint32_t w = lut4k[t];
    return diff >= 0 ? 65535u : w;
}

// exp_attn of a record's (previous max - score) < 0
__device__ __forceinline__ uint32_t exp_rec(int diff, const uint16_t *lut4k, uint32_t c8) {
    const uint32_t neg = 0u - (uint32_t)diff;
    return lut4k[min((uint32_t)(((unsigned long long)neg * c8 + 0x80000000ull) >> 32), 4096u)];
}

// score = round_even(round_even(dot / 4) * mult / 2^15) saturated to int32
// (attention.rs:236-245).  round_even(x / 2^s) = (x + 2^(s-1) - 1 + ((x >> s) & 1)) >> s.
template <bool SAT>
__device__ __forceinline__ int score_from_dot(int dot, int mult) {
    const int du = (dot + 1 + ((dot >> 2) & 1)) >> 2;
    const long long p = (long long)du * (long long)mult;
    long long s = (p + 16383 + ((p >> 15) & 1)) >> 15;
    if (SAT) {   // |mult| >= 2^28: the result may leave the int32 range
        s = s < -2147483648ll ? -2147483648ll : (s > 2147483647ll ? 2147483647ll : s);
    }
    return (int)s;
}

// The same for |mult| < 2^27 with one 64-bit product: X = (du << 13) * (mult << 4) + 2^31
// = 2^17 * (du * mult + 2^14), so the high word of X is floor((du * mult + 2^14) / 2^15),
// the round-half-up quotient, and the low word is zero exactly on a tie, where
// round-half-even takes the even one of the two candidates.  |du| <= 64*127^2/4 < 2^18
// keeps du << 13 inside int32; the score stays inside +-2^30.
__device__ __forceinline__ int score_fast(int dot, int mult16) {
    const int du = (dot + 1 + ((dot >> 2) & 1)) >> 2;
    const long long X = (long long)(du * 8192) * (long long)mult16 + 0x80000000ll;
    const int hi = (int)(X >> 32);
    return (uint32_t)X == 0u ? (hi & ~1) : hi;
}

// Exact scores and exp indices in FP32 (|mult| < 2^19).  A float in [2^23, 2^24) has
// spacing 1, and one fused multiply-add rounds its exact result to nearest, ties to
// even -- the reference's round-half-to-even shift.  With M1 = 1.5 * 2^23 as a bias:
//   bits(M1) + dot              = M1 + dot                     (|dot| < 2^21)
//   fma(M1 + dot, 1/4, 0.75 M1)  = M1 + rne(dot / 4)
//   fma(M1 + du, mult / 2^15, M1 - M1 mult / 2^15) = M1 + rne(du * mult / 2^15)
// (|du * mult / 2^15| < 2^22; mult / 2^15 and M1 - 384 mult are exact floats), so the
// bits of the result minus bits(M1) are the score (attention.rs:236-245), and the bits
// order like the scores.  The exp index t256 = floor((neg * 378194 + 2^23) / 2^24) of a
// difference neg < 2^23 is fma(neg, 378194 / 2^24, M1) - M1 (no ties below 2^22; above
// it the index is clamped at 4096 either way).  Checked exhaustively on the host.
// dot_b: kM1Bits + dot (the QK accumulators start at kM1Bits in MODE 0)
__device__ __forceinline__ int score_flt(int dot_b, float mf, float c2) {
    const float ub = __fmaf_rn(__int_as_float(dot_b), 0.25f, 9437184.0f);
    return __float_as_int(__fmaf_rn(ub, mf, c2));   // biased: kM1Bits + score
}
// t256 of a (non-negative) difference of two biased scores, clamped at 4096 (the
// bias removal and the clamp as one fused add-min)
__device__ __forceinline__ uint32_t t256_flt(int pm_b, int sc_b) {
    const float neg = __fsub_rn(__int_as_float(pm_b), __int_as_float(sc_b));   // exact
    const int tb = __float_as_int(__fmaf_rn(neg, 378194.0f / 16777216.0f, 12582912.0f));
    return (uint32_t)__viaddmin_s32(tb, -(int)kM1Bits, 4096);
}

// One rescale of a state value by a record's factor e (attention.rs:252-259):
// R(x) = (x*e + 2^15) >> 16 for x >= 0, (x*e - 2^15) >> 16 for x < 0
//      = floor((x*e + 2^15) / 2^16) - [x < 0].
// With e16 = e << 16 and x taken as unsigned (x + 2^32 when negative), the high word
// of x*e16 + 2^31 is floor((x*e + 2^15) / 2^16) + [x < 0]*e16, so
// R(x) = hi - [x < 0]*(e16 + 1) (mod 2^32).
__device__ __forceinline__ uint32_t rescale_rec(uint32_t x, uint32_t e16, uint32_t e16p1) {
    const uint32_t h = (uint32_t)(((unsigned long long)x * e16 + 0x80000000ull) >> 32);
    return h + (uint32_t)((int)x >> 31) * e16p1;
}

// key (within a 32-key tile) of QK accumulator column n = 8j + c: accumulator
// entry (j, e) of thread t is key 8t + 2j + e, so each thread holds 8
// consecutive keys and the P*V K index of key 8t + b is 16*(b >> 2) + 4t + (b & 3),
// which the V^T staging turns into storage position 8t + b = the key itself.
__device__ __forceinline__ int perm_key(int n) {
    const int j = n >> 3, c = n & 7;
    return 8 * (c >> 1) + 2 * j + (c & 1);
}

struct Tile {
    uint32_t w[8];    // weights of the row's 8 entries (keys kb + 8t + i)
    uint32_t ef[8];   // (previous max - score) of a record (never 0); other entries: not read
                      // (MODE 0 keeps the difference there, the other modes 0)
    uint32_t rm;      // records among this thread's entries (bit i = entry i)
    uint32_t rowmask; // records of the row in this tile (bit k = key kb + k)
};

// Scores, prefix max, records and weights of row g in one 32-key tile.
// MODE 0: scores in FP32 (|mult| < 2^19), scores and the running max m biased by kM1Bits;
// MODE 1: |mult| < 2^27 (score_fast); MODE 2: any mult (64-bit, saturating).
template <bool MASKED, int MODE, bool EXP0>
__device__ __forceinline__ void tile_softmax(const int (&sacc)[4][4], int kb, int prow, int n, int mult, float mf,
                                             float c2, int t, int &m, const uint16_t *lut4k, uint32_t c8, Tile &T) {
    int sc[8];
    uint32_t rm = 0;
    if constexpr (MODE == 0) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            sc[i] = valid ? score_flt(sacc[i >> 1][i & 1], mf, c2) : INT32_MIN;
        }
        const int x = __vimax3_s32(__vimax3_s32(sc[0], sc[1], sc[2]), __vimax3_s32(sc[3], sc[4], sc[5]),
                                   max(sc[6], sc[7]));
        const int y1 = __shfl_up_sync(0xffffffffu, x, 1, 4);
        const int y2 = __shfl_up_sync(0xffffffffu, x, 2, 4);
        const int y3 = __shfl_up_sync(0xffffffffu, x, 3, 4);
        const int z1 = max(x, __shfl_xor_sync(0xffffffffu, x, 1));
        const int run = m;
        int pm = run;
        if (t >= 1) pm = max(pm, y1);
        if (t >= 2) pm = max(pm, y2);
        if (t >= 3) pm = max(pm, y3);
        if (pm == INT32_MIN) pm = sc[0];
        // an entry is a record iff (prefix max - score) < 0; its sign bits are shifted into
        // rm in entry order (a funnel shift each), reversed once at the end.  The
        // difference itself is kept for every entry: only records' values are read.
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            int ef = pm - sc[i];
            if (MASKED) ef = valid ? ef : 0;
            pm = max(pm, sc[i]);
            uint32_t w = lut4k[t256_flt(pm, sc[i])];
            if (!EXP0) w = pm == sc[i] ? 65535u : w;
            T.w[i] = valid ? w : 0u;
            T.ef[i] = (uint32_t)ef;
            rm = __funnelshift_l((uint32_t)ef, rm, 1);
        }
        rm = __brev(rm) >> 24;
        m = max(run, max(z1, __shfl_xor_sync(0xffffffffu, z1, 2)));
    } else if constexpr (MODE == 1) {
        // |scores| < 2^30, so every difference below fits int32.  The running max is
        // chained from the quad prefix; a record is an entry whose score beats it.
        const int mult16 = mult * 16;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            sc[i] = valid ? score_fast(sacc[i >> 1][i & 1], mult16) : INT32_MIN;
        }
        const int x = max(max(max(sc[0], sc[1]), max(sc[2], sc[3])), max(max(sc[4], sc[5]), max(sc[6], sc[7])));
        const int y1 = __shfl_up_sync(0xffffffffu, x, 1, 4);
        const int y2 = __shfl_up_sync(0xffffffffu, x, 2, 4);
        const int y3 = __shfl_up_sync(0xffffffffu, x, 3, 4);
        const int z1 = max(x, __shfl_xor_sync(0xffffffffu, x, 1));
        const int run = m;
        int pm = run;
        if (t >= 1) pm = max(pm, y1);
        if (t >= 2) pm = max(pm, y2);
        if (t >= 3) pm = max(pm, y3);
        // nothing before it: the row's first key, whose record over INT32_MIN rescales nothing
        if (pm == INT32_MIN) pm = sc[0];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            int ef = min(pm - sc[i], 0);
            if (MASKED) ef = valid ? ef : 0;
            pm = max(pm, sc[i]);
            const uint32_t neg = (uint32_t)pm - (uint32_t)sc[i];
            uint32_t w = lut4k[min((uint32_t)(((unsigned long long)neg * c8 + 0x80000000ull) >> 32), 4096u)];
            if (!EXP0) w = neg == 0u ? 65535u : w;
            T.w[i] = valid ? w : 0u;
            T.ef[i] = (uint32_t)ef;
            rm |= ((uint32_t)ef >> (31 - i)) & (1u << i);
        }
        m = max(run, max(z1, __shfl_xor_sync(0xffffffffu, z1, 2)));
    } else {
        int L[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            sc[i] = valid ? score_from_dot<true>(sacc[i >> 1][i & 1], mult) : INT32_MIN;
            L[i] = i ? max(L[i - 1], sc[i]) : sc[i];   // MODE 2
        }
        // exclusive prefix max over the quad: three independent shuffles
        const int x = L[7];
        const int y1 = __shfl_up_sync(0xffffffffu, x, 1, 4);
        const int y2 = __shfl_up_sync(0xffffffffu, x, 2, 4);
        const int y3 = __shfl_up_sync(0xffffffffu, x, 3, 4);
        const int z1 = max(x, __shfl_xor_sync(0xffffffffu, x, 1));
        const int run = m;
        int base = run;
        if (t >= 1) base = max(base, y1);
        if (t >= 2) base = max(base, y2);
        if (t >= 3) base = max(base, y3);
        int prevmax = base;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            bool valid = true;
            if (MASKED) valid = kb + 8 * t + i <= prow && prow < n;
            const int pm = max(base, L[i]);
            const uint32_t w = exp_attn((int)((uint32_t)sc[i] - (uint32_t)pm), lut4k, c8);
            T.w[i] = valid ? w : 0u;
            // saturated scores may equal INT32_MIN: a record over INT32_MIN rescales nothing
            const bool rec = valid && sc[i] > prevmax && prevmax != INT32_MIN;
            T.ef[i] = rec ? (uint32_t)prevmax - (uint32_t)sc[i] : 0u;
            rm |= rec ? 1u << i : 0u;
            prevmax = pm;
        }
        m = max(run, max(z1, __shfl_xor_sync(0xffffffffu, z1, 2)));
    }
    T.rm = rm;
    uint32_t rowm = rm << (8 * t);
    rowm |= __shfl_xor_sync(0xffffffffu, rowm, 1);
    T.rowmask = rowm | __shfl_xor_sync(0xffffffffu, rowm, 2);
}

// bits 0..3 of x to bit 0 of bytes 0..3
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return ((x & 0xFu) * 0x00204081u) & 0x01010101u; }

// Record bookkeeping of a tile with records.  Segment of each entry (records of
// its row at or before it in key order, at most 32), one byte per entry plus 0x80:
// word q holds entries 4q..4q+3.  The entries' (previous max - score) go to
// rec_e[row][key] (0 where no record); rem[e] = the record mask of PV row 2t+e,
// which the folds walk.
__device__ __forceinline__ void tile_records(const Tile &T, int t, int g, uint32_t *rec_e, uint32_t (&segb)[2],
                                             uint32_t (&rem)[2]) {
    const uint32_t before = (uint32_t)__popc(T.rowmask & ((1u << (8 * t)) - 1u));
    const uint32_t s0 = (spread4(T.rm) + before) * 0x01010101u;
    segb[0] = s0 + 0x80808080u;
    segb[1] = (spread4(T.rm >> 4) + (s0 >> 24)) * 0x01010101u + 0x80808080u;
    uint4 *dst = reinterpret_cast<uint4 *>(rec_e + g * 32 + 8 * t);
    dst[0] = make_uint4(T.ef[0], T.ef[1], T.ef[2], T.ef[3]);
    dst[1] = make_uint4(T.ef[4], T.ef[5], T.ef[6], T.ef[7]);
    rem[0] = __shfl_sync(0xffffffffu, T.rowmask, 8 * t);       // a lane of row 2t's quad
    rem[1] = __shfl_sync(0xffffffffu, T.rowmask, 8 * t + 4);   // row 2t+1
}

// 0xFF in each byte whose segment is >= p, else 0 (segb as tile_records writes it,
// p <= 64): each byte 0x80 + seg - p stays in 64..192, so no borrow crosses bytes and
// bit 7 is set exactly when seg >= p; prmt replicates it over the byte.  The entries
// of segment p are then seg_ge(p) & ~seg_ge(p + 1).
__device__ __forceinline__ uint32_t seg_ge(uint32_t segb, uint32_t p) {
    return prmt(segb - p * 0x01010101u, 0u, 0xBA98u);
}

// One record pass of a tile (attention.rs:248-263): the rows with a pass-th record
// rescale their state by that record's factor, then every row adds its entries of
// segment `pass` (a row with fewer records has none there).  A row's state is
// 256 * hiacc + loacc (mod 2^32) and s_state + 256 * shs + sls: the pass first folds
// every hiacc into its loacc, so the rescale reads one word and the pass's high-byte
// products start from a zero accumulator.  s < 2^32 holds for up to 65,536 keys and a
// sink (65,537 weights <= 65,535: 2^32 - 1), so its rescale is the high word of one
// 64-bit product.
template <int MODE>
__device__ __forceinline__ void record_pass(int pass, int t, uint32_t (&rem)[2], const uint32_t *rec_e,
                                            const uint16_t *lut4k, uint32_t c8, uint32_t (&s_state)[2],
                                            int (&shs)[4], int (&sls)[4], int (&hiacc)[4][4], int (&loacc)[4][4],
                                            const uint32_t (&segb)[2], uint32_t (&geq)[2],
                                            const uint32_t (&phi)[2], const uint32_t (&plo)[2],
                                            const uint32_t (&va)[4][4], const uint32_t (&ones)[4]) {
#pragma unroll
    for (int mi = 0; mi < 4; mi++)
#pragma unroll
        for (int k = 0; k < 4; k++) loacc[mi][k] = (int)(((uint32_t)hiacc[mi][k] << 8) + (uint32_t)loacc[mi][k]);
#pragma unroll
    for (int e = 0; e < 2; e++) {
        if (rem[e] != 0u) {
            const int key = __ffs(rem[e]) - 1;
            rem[e] &= rem[e] - 1u;
            // saturated (MODE 2) scores can wrap the difference to >= 0, where exp gives 65535
            const int rd = (int)rec_e[(2 * t + e) * 32 + key];
            const uint32_t ef = MODE == 2 ? exp_attn(rd, lut4k, c8) : exp_rec(rd, lut4k, c8);
            const uint32_t e16 = ef << 16, e16p1 = e16 + 1u;
            const uint32_t sa = 256u * (uint32_t)shs[e] + (uint32_t)sls[e];
            // s + sa >= 0: R(s + sa) is the high word alone
            s_state[e] = (uint32_t)(((unsigned long long)(s_state[e] + sa) * e16 + 0x80000000ull) >> 32) - sa;
#pragma unroll
            for (int mi = 0; mi < 4; mi++)
#pragma unroll
                for (int k = e; k < 4; k += 2) loacc[mi][k] = (int)rescale_rec((uint32_t)loacc[mi][k], e16, e16p1);
        }
    }
    // P^T of this pass: bytes of entries in segment `pass` (geq: segment >= pass)
    const uint32_t n0 = seg_ge(segb[0], (uint32_t)pass + 1u), n1 = seg_ge(segb[1], (uint32_t)pass + 1u);
    const uint32_t bh0 = phi[0] & geq[0] & ~n0, bl0 = plo[0] & geq[0] & ~n0;
    const uint32_t bh1 = phi[1] & geq[1] & ~n1, bl1 = plo[1] & geq[1] & ~n1;
    geq[0] = n0;
    geq[1] = n1;
    mma_s8u8(shs, ones, bh0, bh1);
    mma_s8u8(sls, ones, bl0, bl1);
#pragma unroll
    for (int mi = 0; mi < 4; mi++) {
        mma_s8u8_z(hiacc[mi], va[mi], bh0, bh1);
        mma_s8u8(loacc[mi], va[mi], bl0, bl1);
    }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

// The 4 KB of one 32-key tile of a stream (K rows, then the V tile) into a
// shared-memory stage, 8 x 16 bytes per lane, as one cp.async group.
__device__ __forceinline__ void decode_tile_async(uint8_t *stage, const int8_t *ks, const int8_t *vt, int kb, int lane) {
#pragma unroll
    for (int i = 0; i < 4; i++) cp_async16(stage + 16 * (lane + 32 * i), ks + (size_t)kb * 64 + 16 * (lane + 32 * i));
#pragma unroll
    for (int i = 0; i < 4; i++)
        cp_async16(stage + 2048 + 16 * (lane + 32 * i), vt + (size_t)kb * 64 + 16 * (lane + 32 * i));
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// STREAM: chunks longer than shared memory holds.  K and V stay in the per-chunk
// streaming layout of k_kv_prep_split (chunk_kvoff[c] * 128 bytes into kv_g) and
// each warp copies its task's 32-key tiles (K rows, then the V tile: 4 KB) into a
// two-stage shared-memory ring with cp.async, the next tile's copy overlapping the
// current tile's work; the fragments then come from the tile as in the decode kernel.
// Nothing of a chunk is staged per CTA, so with gtask given the STREAM kernel is
// persistent: every warp of the grid takes tasks from one counter in global memory
// (gtask, zero at launch), chunk by chunk (longest chunks first) and in each chunk
// longest rows first, task t = (chunk t / (rb_max H), row block rb_max - 1 -
// (t mod rb_max H) / H, head t mod H); row blocks beyond a shorter chunk's end are
// empty tasks.  Only the two or three chunks the warps are on are read at a time, so
// their K/V stay in L2, and no SM idles in a last round of CTAs.  Without gtask, one
// CTA per chunk as the staged kernel.
template <int MODE, bool EXP0, bool STREAM>
__global__ void __launch_bounds__(AM_THREADS, 1)
k_attention_mma(const int8_t *__restrict__ qkv, int ldq, const int8_t *__restrict__ kv_g,
                const int *__restrict__ chunk_row0, const int *__restrict__ chunk_len, int n_heads,
                const int32_t *__restrict__ score_mult, const int8_t *__restrict__ sink_key,
                const int16_t *__restrict__ rope_cos, const int16_t *__restrict__ rope_sin,
                const uint16_t *__restrict__ lut4k_g, int8_t *__restrict__ out, int ldo,
                const int *__restrict__ chunk_kvoff, int *__restrict__ gtask, int n_chunks, int rb_max) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int task_ctr;
    const bool queue = STREAM && gtask != nullptr;   // persistent, global task queue
    int c = queue ? 0 : blockIdx.x;
    int r0 = chunk_row0[c], n = chunk_len[c];
    int npad = (n + 31) & ~31;
    const int vt_ld = ((npad + 127) & ~127) + 32;   // 8 dims of a fragment land on distinct banks
    uint8_t *ks = smem;                              // [npad][64], dims permuted per thread quarter
    uint8_t *vt = ks + npad * 64;                    // [64][vt_ld], keys in order
    uint8_t *wsm = STREAM ? smem : vt + 64 * vt_ld;
    uint16_t *lut_s = reinterpret_cast<uint16_t *>(wsm + AM_WARPS * AM_WARP_SMEM);   // exp table
    for (int i = threadIdx.x; i < AM_LUT; i += AM_THREADS) lut_s[i] = lut4k_g[i];
    const uint16_t *lut4k = lut_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    uint32_t *rec_e = reinterpret_cast<uint32_t *>(wsm + warp * AM_WARP_SMEM);   // [8][32]
    uint8_t *ostage = reinterpret_cast<uint8_t *>(rec_e + AM_ROWS * 32);         // [8][64]
    // STREAM: this warp's two 4 KB tile stages, and the chunk's K rows / V tiles in global memory
    uint8_t *ring = reinterpret_cast<uint8_t *>(lut_s + AM_LUT) + warp * 8192;
    const int8_t *kg = STREAM ? kv_g + (size_t)chunk_kvoff[c] * 128 : nullptr;
    const int8_t *vg = STREAM ? kg + (size_t)npad * 64 : nullptr;
    const int per_chunk = rb_max * n_heads;   // STREAM: tasks per chunk in the global order
    const int g_tasks = n_chunks * per_chunk;

    // K row layout: bytes [16t' + 4k + b] = dim 16k + 4t' + b, so thread t reads its
    // four B words (dims 4t, 16+4t, 32+4t, 48+4t) as one 16-byte load.
    for (int i = tid; i < (STREAM ? 0 : npad * 16); i += AM_THREADS) {
        const int key = i >> 4, wk = i & 15;   // source word: dims 4*wk .. 4*wk+3
        uint32_t v = 0, kw = 0;
        if (key < n) {
            const int8_t *src = kv_g + (size_t)(r0 + key) * 128;
            kw = *reinterpret_cast<const uint32_t *>(src + 4 * wk);
            v = *reinterpret_cast<const uint32_t *>(src + 64 + 4 * wk);
        }
        const int kq = wk >> 2, tq = wk & 3;   // dims 16*kq + 4*tq ..
        *reinterpret_cast<uint32_t *>(ks + key * 64 + 16 * tq + 4 * kq) = kw;
#pragma unroll
        for (int b = 0; b < 4; b++) vt[(4 * wk + b) * vt_ld + key] = (uint8_t)(v >> (8 * b));
    }
    if (tid == 0) task_ctr = 0;
    __syncthreads();

    const uint32_t c8 = 378194u << 8;   // ATTN_COEF_Q24 (attention.rs:14-19) << 8
    const uint32_t ones[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
    const int n_rb = (n + AM_ROWS - 1) / AM_ROWS;
    const int n_tasks = n_rb * n_heads;
    // STREAM: the warp takes AM_TASK_BATCH consecutive tasks per atomic (fewer round
    // trips to one counter), and lane 0 reserves its next batch while the current one runs
    int base = 0, sub = AM_TASK_BATCH;
    int next = (queue && lane == 0) ? atomicAdd(gtask, AM_TASK_BATCH) : 0;
    for (;;) {
        int task = 0, rb, h;
        if (queue) {
            if (sub == AM_TASK_BATCH) {
                base = __shfl_sync(0xffffffffu, next, 0);
                sub = 0;
                if (lane == 0) next = atomicAdd(gtask, AM_TASK_BATCH);
            }
            task = base + sub++;
            if (task >= g_tasks) break;
            c = task / per_chunk;
            const int u = task - c * per_chunk;
            n = chunk_len[c];
            r0 = chunk_row0[c];
            const int kvoff = chunk_kvoff[c];
            rb = rb_max - 1 - u / n_heads;   // longest rows first
            if (rb >= (n + AM_ROWS - 1) / AM_ROWS) continue;   // beyond this chunk's end
            h = u % n_heads;
            npad = (n + 31) & ~31;
            kg = kv_g + (size_t)kvoff * 128;
            vg = kg + (size_t)npad * 64;
        } else {
            if (lane == 0) task = atomicAdd(&task_ctr, 1);
            task = __shfl_sync(0xffffffffu, task, 0);
            if (task >= n_tasks) break;
            rb = n_rb - 1 - task / n_heads;   // longest rows first
            h = task % n_heads;
        }
        const int p0 = rb * AM_ROWS;
        const int prow = p0 + g;                     // the QK / softmax row of this thread
        const int p_last = min(p0 + AM_ROWS - 1, n - 1);
        const bool full_rows = p0 + AM_ROWS - 1 < n;
        const int mult = score_mult[h];
        const float mf = __int2float_rn(mult) * (1.0f / 32768.0f);   // exact (MODE 0)
        const float c2 = __int2float_rn(384 * (32768 - mult));        // M1 - M1 * mf, exact (MODE 0)

        // Q fragment of row g with RoPE (attention.rs:53-83); pairs (i, i+32) live in kk = 0 / 1
        uint32_t qa[2][4];
        {
            uint32_t raw[4] = {0, 0, 0, 0};   // dims 4t, 16+4t, 32+4t, 48+4t (+0..3)
            if (prow < n) {
                const int8_t *qr = qkv + (size_t)(r0 + prow) * ldq + h * 64;
#pragma unroll
                for (int k = 0; k < 4; k++) raw[k] = *reinterpret_cast<const uint32_t *>(qr + 16 * k + 4 * t);
            }
            uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
            for (int k = 0; k < 2; k++)
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    const int i = 16 * k + 4 * t + b;   // dim in 0..31; partner i + 32
                    int x = sext8(raw[k], b), y = sext8(raw[k + 2], b);
                    int cs = 0, sn = 0;
                    if (prow < n) { cs = rope_cos[prow * kHalfDim + i]; sn = rope_sin[prow * kHalfDim + i]; }
                    int xr = rope_q_round(x * cs - y * sn);
                    int yr = rope_q_round(x * sn + y * cs);
                    lo[k] |= (uint32_t)(uint8_t)xr << (8 * b);
                    hi[k] |= (uint32_t)(uint8_t)yr << (8 * b);
                }
            qa[0][0] = lo[0];
            qa[0][2] = lo[1];
            qa[1][0] = hi[0];
            qa[1][2] = hi[1];
            qa[0][1] = qa[0][3] = qa[1][1] = qa[1][3] = 0u;   // A rows 8..15
        }

        int m = INT32_MIN;   // running max of row g
        // PV layout: thread (g, t) holds rows 2t + e, dims 16*mi + g + 8*dh at [mi][2*dh + e]
        uint32_t s_state[2] = {0u, 0u};   // exact in 32 bits (record_pass)
        if (sink_key != nullptr) {   // attention.rs:211-224
            int accs[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                uint32_t b0 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 4 * t);
                uint32_t b1 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 16 + 4 * t);
                mma_s8s8(accs, qa[kk], b0, b1);   // every B column is the sink key
            }
            m = score_from_dot<true>(accs[0], mult);
            if (MODE == 0) m = (int)(kM1Bits + (uint32_t)m);   // biased like the FP32 scores
            s_state[0] = s_state[1] = 65535u;
        }
        int hiacc[4][4], loacc[4][4];
#pragma unroll
        for (int mi = 0; mi < 4; mi++)
#pragma unroll
            for (int k = 0; k < 4; k++) { hiacc[mi][k] = 0; loacc[mi][k] = 0; }
        int shs[4] = {0, 0, 0, 0}, sls[4] = {0, 0, 0, 0};   // weight sums of rows 2t, 2t+1 in [0], [1]

        if (STREAM) decode_tile_async(ring, kg, vg, 0, lane);   // the task's tile 0 in flight
        for (int kb = 0; kb <= p_last; kb += 32) {
            const uint8_t *kst = ks + kb * 64;   // K rows of the tile
            if (STREAM) {   // the next tile's copy overlaps this tile's work; then wait for this one
                if (kb + 32 <= p_last) {
                    decode_tile_async(ring + (((kb >> 5) + 1) & 1) * 4096, kg, vg, kb + 32, lane);
                    asm volatile("cp.async.wait_group 1;" ::: "memory");
                } else {
                    asm volatile("cp.async.wait_group 0;" ::: "memory");
                }
                __syncwarp();
                kst = ring + ((kb >> 5) & 1) * 4096;
            }
            // ---- S = Q K^T over 32 keys (permuted columns) ----
            int sacc[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = MODE == 0 ? (int)kM1Bits : 0;
                const uint4 kw = *reinterpret_cast<const uint4 *>(kst + perm_key(8 * j + g) * 64 + 16 * t);
                mma_s8s8(sacc[j], qa[0], kw.x, kw.y);
                mma_s8s8(sacc[j], qa[1], kw.z, kw.w);
            }
            // V^T A fragments: dims 16mi+g / +8; K 4t.. (word 0) and 16+4t.. (word 1) = keys 8t..8t+7
            uint32_t va[4][4];
            if (STREAM) {   // V tile, lane-major (vt_byte): the lane's 16 words as four 16-byte loads
                const uint4 *vl = reinterpret_cast<const uint4 *>(kst + 2048) + 4 * lane;
#pragma unroll
                for (int mi = 0; mi < 4; mi++) {
                    const uint4 v = vl[mi ^ ((lane >> 1) & 3)];
                    va[mi][0] = v.x; va[mi][1] = v.y; va[mi][2] = v.z; va[mi][3] = v.w;
                }
                __syncwarp();   // every lane has its fragments: the stage may be refilled next tile
            } else {
#pragma unroll
                for (int mi = 0; mi < 4; mi++) {
                    const uint2 lo2 = *reinterpret_cast<const uint2 *>(vt + (16 * mi + g) * vt_ld + kb + 8 * t);
                    const uint2 hi2 = *reinterpret_cast<const uint2 *>(vt + (16 * mi + g + 8) * vt_ld + kb + 8 * t);
                    va[mi][0] = lo2.x;
                    va[mi][1] = hi2.x;
                    va[mi][2] = lo2.y;
                    va[mi][3] = hi2.y;
                }
            }

            Tile T;
            if (!full_rows || kb + 31 > p0)
                tile_softmax<true, MODE, EXP0>(sacc, kb, prow, n, mult, mf, c2, t, m, lut4k, c8, T);
            else
                tile_softmax<false, MODE, EXP0>(sacc, kb, prow, n, mult, mf, c2, t, m, lut4k, c8, T);
            // P^T B fragments (u8 halves of the weights): word q = entries 4q..4q+3
            uint32_t phi[2], plo[2];
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint32_t x01 = prmt(T.w[4 * q], T.w[4 * q + 1], 0x5140u);   // lo0 lo1 hi0 hi1
                const uint32_t x23 = prmt(T.w[4 * q + 2], T.w[4 * q + 3], 0x5140u);
                plo[q] = prmt(x01, x23, 0x5410u);
                phi[q] = prmt(x01, x23, 0x7632u);
            }
            const int maxrec = (int)__reduce_max_sync(0xffffffffu, (unsigned)__popc(T.rowmask));
            uint32_t segb[2] = {0, 0}, geq[2] = {0, 0};
            uint32_t rem[2] = {0, 0};   // records of the PV rows 2t, 2t+1 not yet folded
            if (maxrec > 0) {
                tile_records(T, t, g, rec_e, segb, rem);
                __syncwarp();
            }
            {   // pass 0: the whole tile, or segment 0 of each row
                uint32_t bh0 = phi[0], bh1 = phi[1], bl0 = plo[0], bl1 = plo[1];
                if (maxrec > 0) {
                    geq[0] = seg_ge(segb[0], 1u);
                    geq[1] = seg_ge(segb[1], 1u);
                    bh0 &= ~geq[0]; bl0 &= ~geq[0]; bh1 &= ~geq[1]; bl1 &= ~geq[1];
                }
                mma_s8u8(shs, ones, bh0, bh1);   // weight sums (all-ones rows)
                mma_s8u8(sls, ones, bl0, bl1);
#pragma unroll
                for (int mi = 0; mi < 4; mi++) {
                    mma_s8u8(hiacc[mi], va[mi], bh0, bh1);
                    mma_s8u8(loacc[mi], va[mi], bl0, bl1);
                }
            }
            for (int pass = 1; pass <= maxrec; pass++) {
                record_pass<MODE>(pass, t, rem, rec_e, lut4k, c8, s_state, shs, sls, hiacc, loacc, segb, geq, phi,
                                  plo, va, ones);
            }
        }

        // output: clamp(round_half_even(vacc / s)) (attention.rs:279-284), staged per warp
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const uint32_t sv = s_state[e] + 256u * (uint32_t)shs[e] + (uint32_t)sls[e];
            const uint32_t den = sv == 0 ? 1u : sv;
            const float rcp = __frcp_rn(__uint2float_rn(den));
            uint8_t *orow = ostage + (2 * t + e) * 64;
#pragma unroll
            for (int mi = 0; mi < 4; mi++)
#pragma unroll
                for (int dh = 0; dh < 2; dh++) {
                    const int k = 2 * dh + e;
                    const int x = (int)(((uint32_t)hiacc[mi][k] << 8) + (uint32_t)loacc[mi][k]);
                    orow[16 * mi + g + 8 * dh] = (uint8_t)div_rne_clamp127(x, den, rcp);
                }
        }
        __syncwarp();
        {   // 8 rows x 4 pieces of 16 bytes: one per lane
            const int row = lane >> 2, part = lane & 3;
            if (p0 + row < n)
                *reinterpret_cast<uint4 *>(out + (size_t)(r0 + p0 + row) * ldo + h * 64 + 16 * part) =
                    *reinterpret_cast<const uint4 *>(ostage + row * 64 + 16 * part);
        }
        __syncwarp();
    }
}

// Decode: one warp per stream r, the query of every head at position p against
// the stream's keys 0..p in the split cache layout (K rows of 64 permuted dims,
// then V in 2 KB tiles of 32 keys in the lane-major layout of vt_byte, common.cuh).  The heads are the 8 rows of the attention tile (A rows
// n_heads..15 are zero); everything else is the chunk kernel's tile step.
// The warp also appends the stream's key p (RoPE) and value p, from columns kd..kd+127
// of its qkv row, to the cache (the layout of k_kv_append, decode.cu) and patches
// them into the stage of the last tile once that tile's copy has landed: the copy may
// have been issued before the row was written.
// Persistent: one CTA per SM, warp w takes streams w, w + W, w + 2W, ... (W the
// warps of the grid).  A warp's tiles, stream after stream, flow through a ring of
// DEC_STAGES 4 KB shared-memory stages with DEC_STAGES - 1 tile copies in flight,
// so the first tiles of the next stream load while the current one finishes; the
// stream's qkv row (its queries and the step's key and value) rides in the copy
// group of its first tile, and the position's RoPE values sit in shared memory.
constexpr int DEC_STAGES = 2;
constexpr int DEC_ROW = 640;   // a stream's qkv row (d + 128 bytes, d <= 512 with at most 8 heads)
constexpr int DEC_SMEM = AM_WARPS * DEC_STAGES * 4096 + AM_LUT * 2 + 128 + AM_WARPS * DEC_ROW;

template <int MODE, bool EXP0>
__global__ void __launch_bounds__(AM_THREADS, 1)
k_attention_decode_mma(const int8_t *__restrict__ qkv, int ldq, int kd, int8_t *kvc, size_t cache_ld,
                       int M, int p, int n_heads, const int32_t *__restrict__ score_mult,
                       const int8_t *__restrict__ sink_key, const int16_t *__restrict__ rope_cos,
                       const int16_t *__restrict__ rope_sin, const uint16_t *__restrict__ lut4k_g,
                       int8_t *__restrict__ out, int ldo) {
    __shared__ __align__(16) uint8_t wsm[AM_WARPS * AM_WARP_SMEM];
    extern __shared__ __align__(16) uint8_t dsm[];   // per warp: DEC_STAGES 4 KB tile stages; then the exp table
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    uint16_t *lut_s = reinterpret_cast<uint16_t *>(dsm + AM_WARPS * DEC_STAGES * 4096);
    for (int i = tid; i < AM_LUT; i += AM_THREADS) lut_s[i] = lut4k_g[i];   // model constant
    // the RoPE values of position p (model constants): cos at [0, 32), sin at [32, 64)
    int16_t *rope_s = reinterpret_cast<int16_t *>(lut_s + AM_LUT);
    if (tid < 2 * kHalfDim) rope_s[tid] = tid < kHalfDim ? rope_cos[p * kHalfDim + tid] : rope_sin[p * kHalfDim + tid - kHalfDim];
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    const uint16_t *lut4k = lut_s;
    const int stride = gridDim.x * AM_WARPS;
    int r = blockIdx.x * AM_WARPS + warp;
    if (r >= M) return;
    uint8_t *stages = dsm + warp * (DEC_STAGES * 4096);
    // this warp's copy of its current stream's qkv row, loaded with the stream's first tile
    uint8_t *qrow = reinterpret_cast<uint8_t *>(rope_s + 2 * kHalfDim) + warp * DEC_ROW;
    const int row_chunks = ldq >> 4;   // ldq = d + 128 <= DEC_ROW, a multiple of 16
    uint32_t *rec_e = reinterpret_cast<uint32_t *>(wsm + warp * AM_WARP_SMEM);   // [8][32]
    uint8_t *ostage = reinterpret_cast<uint8_t *>(rec_e + AM_ROWS * 32);         // [8][64]
    const size_t len = cache_ld / 128;
    const uint32_t c8 = 378194u << 8;   // ATTN_COEF_Q24 (attention.rs:14-19) << 8
    const uint32_t ones[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
    const bool head = g < n_heads;   // row g of the tile is head g
    const int mult = head ? score_mult[g] : 0;
    const float mf = __int2float_rn(mult) * (1.0f / 32768.0f);
    const float c2 = __int2float_rn(384 * (32768 - mult));
    const int ntiles = (p >> 5) + 1;

    // the tile sequence (stream fr, tile fk), its next copy going to stage fslot;
    // past the warp's last tile an empty group keeps the group count in step
    int fr = r, fk = 0, fslot = 0, cslot = 0;
    auto fetch = [&]() {
        if (fr < M) {
            const int8_t *k0 = kvc + (size_t)fr * cache_ld;   // [len][64] K rows, then the V tiles
            if (fk == 0)   // the stream's qkv row joins its first tile's copy group
                for (int c = lane; c < row_chunks; c += 32) cp_async16(qrow + 16 * c, qkv + (size_t)fr * ldq + 16 * c);
            decode_tile_async(stages + fslot * 4096, k0, k0 + len * 64, 32 * fk, lane);
            if (++fk == ntiles) { fk = 0; fr += stride; }
        } else {
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        fslot = fslot + 1 == DEC_STAGES ? 0 : fslot + 1;
    };
#pragma unroll
    for (int i = 0; i < DEC_STAGES - 1; i++) fetch();

    for (; r < M; r += stride) {

    // this stream's qkv row (and first tile) have landed: the only copy group in flight
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    // Q fragment of head g at position p with RoPE (attention.rs:53-83)
    uint32_t qa[2][4];
    {
        uint32_t raw[4] = {0, 0, 0, 0};
        if (head) {
            const uint8_t *qr = qrow + g * 64;
#pragma unroll
            for (int k = 0; k < 4; k++) raw[k] = *reinterpret_cast<const uint32_t *>(qr + 16 * k + 4 * t);
        }
        uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
        for (int k = 0; k < 2; k++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int i = 16 * k + 4 * t + b;
                int x = sext8(raw[k], b), y = sext8(raw[k + 2], b);
                const int cs = rope_s[i], sn = rope_s[kHalfDim + i];
                int xr = rope_q_round(x * cs - y * sn);
                int yr = rope_q_round(x * sn + y * cs);
                lo[k] |= (uint32_t)(uint8_t)xr << (8 * b);
                hi[k] |= (uint32_t)(uint8_t)yr << (8 * b);
            }
        qa[0][0] = lo[0];
        qa[0][2] = lo[1];
        qa[1][0] = hi[0];
        qa[1][2] = hi[1];
        qa[0][1] = qa[0][3] = qa[1][1] = qa[1][3] = 0u;
    }
    // key p rotated (attention.rs:29-50) and value p: lane l holds dims l, l + 32 of the
    // key and dims 2l, 2l + 1 of the value, written to the cache now and kept (one word
    // per lane, in the output staging area, free until the output) for the last tile
    {
        const int8_t *kq = reinterpret_cast<const int8_t *>(qrow) + kd;
        const int x = kq[lane], y = kq[lane + kHalfDim];
        const int cs = rope_s[lane], sn = rope_s[kHalfDim + lane];
        const int kx = rope_k_round(x * cs - y * sn);
        const int ky = rope_k_round(x * sn + y * cs);
        const uint32_t v2 = *reinterpret_cast<const uint16_t *>(kq + 64 + 2 * lane);
        reinterpret_cast<uint32_t *>(ostage)[lane] = (uint32_t)(uint8_t)kx | ((uint32_t)(uint8_t)ky << 8) | (v2 << 16);
        int8_t *base = kvc + (size_t)r * cache_ld;
        const int l2 = lane + kHalfDim;
        base[(size_t)p * 64 + 16 * ((lane >> 2) & 3) + 4 * (lane >> 4) + (lane & 3)] = (int8_t)kx;
        base[(size_t)p * 64 + 16 * ((l2 >> 2) & 3) + 4 * (l2 >> 4) + (l2 & 3)] = (int8_t)ky;
        int8_t *vt = base + len * 64 + (size_t)(p >> 5) * 2048;   // the V tile of key p
        vt[vt_byte(p & 31, 2 * lane)] = (int8_t)(v2 & 0xFFu);
        vt[vt_byte(p & 31, 2 * lane + 1)] = (int8_t)(v2 >> 8);
    }
    __syncwarp();   // every lane has read the row: the next stream's copy may overwrite it
    int m = INT32_MIN;
    uint32_t s_state[2] = {0u, 0u};   // exact in 32 bits (record_pass)
    if (sink_key != nullptr) {   // attention.rs:211-224
        int accs[4] = {0, 0, 0, 0};
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
            uint32_t b0 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 4 * t);
            uint32_t b1 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 16 + 4 * t);
            mma_s8s8(accs, qa[kk], b0, b1);
        }
        m = score_from_dot<true>(accs[0], mult);
        if (MODE == 0) m = (int)(kM1Bits + (uint32_t)m);
        s_state[0] = s_state[1] = 65535u;
    }
    int hiacc[4][4], loacc[4][4];
#pragma unroll
    for (int mi = 0; mi < 4; mi++)
#pragma unroll
        for (int k = 0; k < 4; k++) { hiacc[mi][k] = 0; loacc[mi][k] = 0; }
    int shs[4] = {0, 0, 0, 0}, sls[4] = {0, 0, 0, 0};

    for (int kb = 0; kb <= p; kb += 32) {
        // keep DEC_STAGES - 1 copies in flight ahead of this tile, then wait for it
        fetch();
        asm volatile("cp.async.wait_group %0;" ::"n"(DEC_STAGES - 1) : "memory");
        __syncwarp();
        uint8_t *kst = stages + cslot * 4096;   // K rows of the tile, then the V tile
        cslot = cslot + 1 == DEC_STAGES ? 0 : cslot + 1;
        if (kb + 32 > p) {   // the last tile: key p and value p from this step
            const uint32_t kvw = reinterpret_cast<const uint32_t *>(ostage)[lane];
            const int l2 = lane + kHalfDim, kp = p & 31;
            kst[kp * 64 + 16 * ((lane >> 2) & 3) + 4 * (lane >> 4) + (lane & 3)] = (uint8_t)kvw;
            kst[kp * 64 + 16 * ((l2 >> 2) & 3) + 4 * (l2 >> 4) + (l2 & 3)] = (uint8_t)(kvw >> 8);
            uint8_t *vs = kst + 2048;
            vs[vt_byte(kp, 2 * lane)] = (uint8_t)(kvw >> 16);
            vs[vt_byte(kp, 2 * lane + 1)] = (uint8_t)(kvw >> 24);
            __syncwarp();
        }
        int sacc[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = MODE == 0 ? (int)kM1Bits : 0;
            const uint4 kw = *reinterpret_cast<const uint4 *>(kst + perm_key(8 * j + g) * 64 + 16 * t);
            mma_s8s8(sacc[j], qa[0], kw.x, kw.y);
            mma_s8s8(sacc[j], qa[1], kw.z, kw.w);
        }
        // V^T A fragments: word (group 2t or 2t+1 = keys 8t..8t+3 / 8t+4..8t+7, dim)
        uint32_t va[4][4];
        const uint4 *vl = reinterpret_cast<const uint4 *>(kst + 2048) + 4 * lane;   // lane-major (vt_byte)
#pragma unroll
        for (int mi = 0; mi < 4; mi++) {
            const uint4 v = vl[mi ^ ((lane >> 1) & 3)];
            va[mi][0] = v.x; va[mi][1] = v.y; va[mi][2] = v.z; va[mi][3] = v.w;
        }
        __syncwarp();   // every lane has its fragments: the stage may be refilled next iteration
        Tile T;
        if (kb + 31 > p)
            tile_softmax<true, MODE, EXP0>(sacc, kb, p, p + 1, mult, mf, c2, t, m, lut4k, c8, T);
        else
            tile_softmax<false, MODE, EXP0>(sacc, kb, p, p + 1, mult, mf, c2, t, m, lut4k, c8, T);
        uint32_t phi[2], plo[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const uint32_t x01 = prmt(T.w[4 * q], T.w[4 * q + 1], 0x5140u);
            const uint32_t x23 = prmt(T.w[4 * q + 2], T.w[4 * q + 3], 0x5140u);
            plo[q] = prmt(x01, x23, 0x5410u);
            phi[q] = prmt(x01, x23, 0x7632u);
        }
        const int maxrec = (int)__reduce_max_sync(0xffffffffu, (unsigned)__popc(T.rowmask));
        uint32_t segb[2] = {0, 0}, geq[2] = {0, 0};
        uint32_t rem[2] = {0, 0};
        if (maxrec > 0) {
            tile_records(T, t, g, rec_e, segb, rem);
            __syncwarp();
        }
        {   // pass 0: the whole tile, or segment 0 of each row
            uint32_t bh0 = phi[0], bh1 = phi[1], bl0 = plo[0], bl1 = plo[1];
            if (maxrec > 0) {
                geq[0] = seg_ge(segb[0], 1u);
                geq[1] = seg_ge(segb[1], 1u);
                bh0 &= ~geq[0]; bl0 &= ~geq[0]; bh1 &= ~geq[1]; bl1 &= ~geq[1];
            }
            mma_s8u8(shs, ones, bh0, bh1);
            mma_s8u8(sls, ones, bl0, bl1);
#pragma unroll
            for (int mi = 0; mi < 4; mi++) {
                mma_s8u8(hiacc[mi], va[mi], bh0, bh1);
                mma_s8u8(loacc[mi], va[mi], bl0, bl1);
            }
        }
        for (int pass = 1; pass <= maxrec; pass++)
            record_pass<MODE>(pass, t, rem, rec_e, lut4k, c8, s_state, shs, sls, hiacc, loacc, segb, geq, phi, plo,
                              va, ones);
    }

    // output of heads 2t, 2t+1 (attention.rs:279-284)
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const uint32_t sv = s_state[e] + 256u * (uint32_t)shs[e] + (uint32_t)sls[e];
        const RneDiv dv = make_rne_div(sv == 0 ? 1ull : sv);   // the integer form measured faster per stream step
        uint8_t *orow = ostage + (2 * t + e) * 64;
#pragma unroll
        for (int mi = 0; mi < 4; mi++)
#pragma unroll
            for (int dh = 0; dh < 2; dh++) {
                const int k = 2 * dh + e;
                const int x = (int)(((uint32_t)hiacc[mi][k] << 8) + (uint32_t)loacc[mi][k]);
                orow[16 * mi + g + 8 * dh] = (uint8_t)clamp127(div_rne_s32_by(x, dv));
            }
    }
    __syncwarp();
    {
        const int hd = lane >> 2, part = lane & 3;
        if (hd < n_heads)
            *reinterpret_cast<uint4 *>(out + (size_t)r * ldo + hd * 64 + 16 * part) =
                *reinterpret_cast<const uint4 *>(ostage + hd * 64 + 16 * part);
    }
    __syncwarp();   // ostage and rec_e are reused by the next stream
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

}  // namespace

size_t attention_mma_smem(int max_len) {
    const int npad = (max_len + 31) & ~31;
    const int vt_ld = ((npad + 127) & ~127) + 32;
    return (size_t)npad * 64 + (size_t)64 * vt_ld + (size_t)AM_WARPS * AM_WARP_SMEM + AM_LUT * 2;
}

bool attention_mma_fits(int max_len) { return max_len <= AM_MAX_KEYS; }

constexpr int AM_STREAM_SMEM = AM_WARPS * AM_WARP_SMEM + AM_LUT * 2 + AM_WARPS * 8192;

void attention_mma_init() {
    cudaFuncSetAttribute(k_attention_decode_mma<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    cudaFuncSetAttribute(k_attention_decode_mma<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    cudaFuncSetAttribute(k_attention_decode_mma<0, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    cudaFuncSetAttribute(k_attention_decode_mma<0, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    cudaFuncSetAttribute(k_attention_decode_mma<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    const int smem = (int)attention_mma_smem(AM_MAX_KEYS);
    cudaFuncSetAttribute(k_attention_mma<1, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention_mma<1, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention_mma<1, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AM_STREAM_SMEM);
    cudaFuncSetAttribute(k_attention_mma<1, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AM_STREAM_SMEM);
    cudaFuncSetAttribute(k_attention_mma<0, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention_mma<0, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention_mma<2, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention_mma<0, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AM_STREAM_SMEM);
    cudaFuncSetAttribute(k_attention_mma<0, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AM_STREAM_SMEM);
    cudaFuncSetAttribute(k_attention_mma<2, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         AM_STREAM_SMEM);
}

void launch_attention_mma(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                          const int *chunk_len, int n_chunks, int max_len, int n_heads,
                          const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                          const int16_t *rope_sin, const uint16_t *lut4k, int score_mode, bool exp0, int8_t *out,
                          int ldo, cudaStream_t st) {
    if (n_chunks == 0) return;
    const size_t smem = attention_mma_smem(max_len);
    if (score_mode == 1) {
        if (exp0)
            k_attention_mma<1, true, false><<<n_chunks, AM_THREADS, smem, st>>>(
                qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
                lut4k, out, ldo, nullptr, nullptr, n_chunks, 0);
        else
            k_attention_mma<1, false, false><<<n_chunks, AM_THREADS, smem, st>>>(
                qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
                lut4k, out, ldo, nullptr, nullptr, n_chunks, 0);
    } else if (score_mode == 2)
        k_attention_mma<2, false, false><<<n_chunks, AM_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, nullptr, nullptr, n_chunks, 0);
    else if (exp0)
        k_attention_mma<0, true, false><<<n_chunks, AM_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, nullptr, nullptr, n_chunks, 0);
    else
        k_attention_mma<0, false, false><<<n_chunks, AM_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, nullptr, nullptr, n_chunks, 0);
}

void launch_attention_mma_stream(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                                 const int *chunk_len, const int *chunk_kvoff, int n_chunks, int max_len, int n_heads,
                                 const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                                 const int16_t *rope_sin, const uint16_t *lut4k, int score_mode, bool exp0,
                                 int8_t *out, int ldo, int *task_ctr, cudaStream_t st) {
    if (n_chunks == 0 || max_len <= 0) return;
    const int rb_max = (max_len + AM_ROWS - 1) / AM_ROWS;
    // the global queue from chunks of 1024 keys on (per 3 M-token sample: ctx 1024
    // -1.9%, ctx 4096 -27%); at ctx 512 its short tasks ran 2-3% slower than one CTA
    // per chunk, whose last round is then a small part of ~20 (CZG_ATTN_QUEUE=0 / 1)
    const char *qe = getenv("CZG_ATTN_QUEUE");
    const bool queue = qe ? qe[0] != '0' : max_len >= 1024;
    int grid = n_chunks;
    if (queue) {
        cudaMemsetAsync(task_ctr, 0, sizeof(int), st);
        const long long tasks = (long long)n_chunks * rb_max * n_heads;
        grid = (int)std::min<long long>((tasks + AM_WARPS - 1) / AM_WARPS, (long long)sm_count());
    } else {
        task_ctr = nullptr;
    }
    if (score_mode == 1) {
        if (exp0)
            k_attention_mma<1, true, true><<<grid, AM_THREADS, AM_STREAM_SMEM, st>>>(
                qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
                lut4k, out, ldo, chunk_kvoff, task_ctr, n_chunks, rb_max);
        else
            k_attention_mma<1, false, true><<<grid, AM_THREADS, AM_STREAM_SMEM, st>>>(
                qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
                lut4k, out, ldo, chunk_kvoff, task_ctr, n_chunks, rb_max);
    } else if (score_mode == 2)
        k_attention_mma<2, false, true><<<grid, AM_THREADS, AM_STREAM_SMEM, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, chunk_kvoff, task_ctr, n_chunks, rb_max);
    else if (exp0)
        k_attention_mma<0, true, true><<<grid, AM_THREADS, AM_STREAM_SMEM, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, chunk_kvoff, task_ctr, n_chunks, rb_max);
    else
        k_attention_mma<0, false, true><<<grid, AM_THREADS, AM_STREAM_SMEM, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo, chunk_kvoff, task_ctr, n_chunks, rb_max);
}

bool attention_decode_mma_ok(int n_heads) { return n_heads >= 1 && n_heads <= AM_ROWS; }

void launch_attention_decode_mma(const int8_t *qkv, int ldq, int kd, int8_t *kvc, size_t cache_ld, int M, int p,
                                 int n_heads, const int32_t *score_mult, const int8_t *sink_key,
                                 const int16_t *rope_cos, const int16_t *rope_sin, const uint16_t *lut4k,
                                 int score_mode, bool exp0, int8_t *out, int ldo, cudaStream_t st) {
    if (M == 0) return;
    const unsigned grid = (unsigned)std::min<long>((M + AM_WARPS - 1) / AM_WARPS, (long)sm_count());
    if (score_mode == 1) {
        if (exp0)
            launch_k(k_attention_decode_mma<1, true>, grid, AM_THREADS, DEC_SMEM, st, qkv, ldq, kd, kvc, cache_ld, M, p,
                     n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k, out, ldo);
        else
            launch_k(k_attention_decode_mma<1, false>, grid, AM_THREADS, DEC_SMEM, st, qkv, ldq, kd, kvc, cache_ld, M, p,
                     n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k, out, ldo);
    } else if (score_mode == 2)
        launch_k(k_attention_decode_mma<2, false>, grid, AM_THREADS, DEC_SMEM, st, qkv, ldq, kd, kvc, cache_ld, M, p,
                 n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k, out, ldo);
    else if (exp0)
        launch_k(k_attention_decode_mma<0, true>, grid, AM_THREADS, DEC_SMEM, st, qkv, ldq, kd, kvc, cache_ld, M, p,
                 n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k, out, ldo);
    else
        launch_k(k_attention_decode_mma<0, false>, grid, AM_THREADS, DEC_SMEM, st, qkv, ldq, kd, kvc, cache_ld, M, p,
                 n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k, out, ldo);
}

}  // namespace czg
