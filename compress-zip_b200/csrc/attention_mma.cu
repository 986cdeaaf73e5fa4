// attention_mma.cu -- exact causal integer attention on the tensor cores.
//
// Same result as rust/src/attention.rs:162-289 run for positions 0..n-1 of a
// chunk (see attention.cu for the scalar form).  Per warp task: 16 query rows
// of one head against all their keys, 32 keys per tile.
//
// QK^T: mma.sync m16n8k32 s8*s8 -> s32 gives the exact int32 dot products.  The
// key order inside a tile is permuted for the QK product so that each thread's
// accumulator entries are exactly the keys its P fragment needs for P*V
// (thread t of a quad holds keys 4t..4t+3 and 16+4t..16+4t+3 of rows g, g+8).
//
// Online softmax: per row, scores -> prefix max in key order (thread-local run
// + quad scan) -> records (keys beating everything before them) -> weights
// w = exp(score - max so far) and rescale factors e = exp(old max - score).
//
// P*V: the 16-bit weights are split into a high and a low byte and multiplied
// with V (s8) as two u8*s8 MMAs into separate accumulators Hi, Lo; each is
// exactly sum(byte * v) and never overflows (|sum| <= 255*127*4096), so
// vacc = 256*Hi + Lo (mod 2^32) equals the reference's wrapping i32 sum.
// A tile whose rows contain records is replayed in passes: pass q adds the keys
// of segment q (segment = run of keys between records).  Before pass q every
// row with a q-th record in the tile folds its state exactly as the reference
// rescales at that key: state = R(state + 256*Hi + Lo, e),
// s = ((s + seg_sum) * e + 2^15) >> 16.  The folded state of a warp's 16 rows
// lives in shared memory as [row][dim] so that all 32 lanes fold one row
// together (2 dims each).
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int AM_THREADS = 256;
constexpr int AM_WARPS = AM_THREADS / 32;
constexpr int AM_MAX_KEYS = 1024;
constexpr int AM_ROW = 72;   // words per row of the per-warp state buffers (bank-spread)
constexpr int AM_WARP_SMEM = 16 * AM_ROW * 4 * 2 + 16 * 32 * 4 + 16 * 4 * 2;   // vst, segbuf, rec_e, nrec, s

__device__ __forceinline__ void mma_s8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// exp_q16 with the attention coefficient via a 4096-entry table indexed by
// t256 (entries for t256 >= 4096 are all 1, whatever the exp2 LUT holds).
// t256 = floor((neg * coef + 2^23) / 2^24) = hi + (lo >= 2^31) of neg * (coef << 8).
__device__ __forceinline__ uint32_t exp_attn(int diff, const uint16_t *lut4k, uint32_t c8) {
    if (diff >= 0) return 65535u;
    uint32_t neg = 0u - (uint32_t)diff;
    uint32_t t = __umulhi(neg, c8) + ((neg * c8) >> 31);
    uint32_t w = 1u;
    if (t < 4096u) w = __ldg(lut4k + t);   // only lanes near the running max touch the table
    return w;
}

// score = round_even(round_even(dot / 4) * mult / 2^15) saturated to int32
// (attention.rs:236-245).  round_even(x / 2^s) = (x + 2^(s-1) - 1 + ((x >> s) & 1)) >> s.
template <bool WIDE>
__device__ __forceinline__ int score_from_dot(int dot, int mult) {
    const int du = (dot + 1 + ((dot >> 2) & 1)) >> 2;
    const long long p = (long long)du * (long long)mult;
    long long s = (p + 16383 + ((p >> 15) & 1)) >> 15;
    if (WIDE) {   // |mult| >= 2^28: the result may leave the int32 range
        s = s < -2147483648ll ? -2147483648ll : (s > 2147483647ll ? 2147483647ll : s);
    }
    return (int)s;
}

// key (within a 32-key tile) of QK accumulator column / B row n = 8j + r
__device__ __forceinline__ int perm_key(int n) {
    int j = n >> 3, r = n & 7;
    return 16 * (j >> 1) + 4 * (r >> 1) + 2 * (j & 1) + (r & 1);
}

struct Tile {
    uint32_t w[2][8];     // weights of each row half's 8 entries
    uint32_t ef[2][8];    // 0, or record flag | rescale factor
    int lrec[2][2];       // records of this thread per row half and 16-key half
    int nrec[2];          // records of the row in this tile (quad total)
};

// Scores, prefix max, records and weights of one 32-key tile.
// Entry i of a row half is key kb + 16*(i>>2) + 4t + (i&3).
template <bool MASKED, bool WIDE>
__device__ __forceinline__ void tile_softmax(const int (&sacc)[4][4], int kb, const int (&prow)[2], int n,
                                             int mult, int t, int lane, int (&m)[2],
                                             const uint16_t *lut4k, uint32_t c8, Tile &T) {
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        int sc[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int q = i >> 2, b = i & 3;
            const int j = 2 * q + (b >> 1), e = b & 1;
            bool valid = true;
            if (MASKED) valid = kb + 16 * q + 4 * t + b <= prow[hr] && prow[hr] < n;
            sc[i] = valid ? score_from_dot<WIDE>(sacc[j][2 * hr + e], mult) : INT32_MIN;
        }
        int run = m[hr];
        int total = 0;
#pragma unroll
        for (int q = 0; q < 2; q++) {
            int L[4];
            L[0] = sc[4 * q];
#pragma unroll
            for (int b = 1; b < 4; b++) L[b] = max(L[b - 1], sc[4 * q + b]);
            int inc = L[3];
            int u = __shfl_up_sync(0xffffffffu, inc, 1, 4);
            if (t >= 1) inc = max(inc, u);
            u = __shfl_up_sync(0xffffffffu, inc, 2, 4);
            if (t >= 2) inc = max(inc, u);
            const int excl = __shfl_up_sync(0xffffffffu, inc, 1, 4);
            const int base = t == 0 ? run : max(run, excl);
            int prevmax = base;
            int lrec = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int i = 4 * q + b;
                bool valid = true;
                if (MASKED) valid = kb + 16 * q + 4 * t + b <= prow[hr] && prow[hr] < n;
                const int pm = max(base, L[b]);
                const bool rec = valid && sc[i] > prevmax;
                T.w[hr][i] = valid ? exp_attn((int)((uint32_t)sc[i] - (uint32_t)pm), lut4k, c8) : 0u;
                uint32_t f = 0;
                if (rec) {
                    // 0x10000 | factor, or 0x20000 while the previous max is still INT32_MIN:
                    // the reference then keeps its sums unscaled (attention.rs:248-250)
                    f = prevmax == INT32_MIN
                            ? 0x20000u
                            : 0x10000u | exp_attn((int)((uint32_t)prevmax - (uint32_t)sc[i]), lut4k, c8);
                    lrec++;
                }
                T.ef[hr][i] = f;
                prevmax = pm;
            }
            T.lrec[hr][q] = lrec;
            total += lrec;
            run = max(run, __shfl_sync(0xffffffffu, inc, (lane & ~3) | 3));
        }
        m[hr] = run;
        total += __shfl_xor_sync(0xffffffffu, total, 1);
        total += __shfl_xor_sync(0xffffffffu, total, 2);
        T.nrec[hr] = total;
    }
}

// Segment of each entry (records at or before it in key order within the tile),
// packed one byte per entry in A-fragment word order (word hr + 2q, byte b); the
// record factors are published to rec_e[row][segment - 1].
__device__ __forceinline__ void tile_segments(const Tile &T, int t, int g, uint32_t *rec_e, int *nrec_s,
                                              uint32_t (&segw)[4]) {
#pragma unroll
    for (int hr = 0; hr < 2; hr++) {
        const int row = g + 8 * hr;
        int before = 0;
#pragma unroll
        for (int q = 0; q < 2; q++) {
            int cinc = T.lrec[hr][q];
            int cu = __shfl_up_sync(0xffffffffu, cinc, 1, 4);
            if (t >= 1) cinc += cu;
            cu = __shfl_up_sync(0xffffffffu, cinc, 2, 4);
            if (t >= 2) cinc += cu;
            int sidx = before + cinc - T.lrec[hr][q];
            uint32_t word = 0;
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int i = 4 * q + b;
                if (T.ef[hr][i]) {
                    sidx++;
                    rec_e[row * 32 + sidx - 1] = T.ef[hr][i];
                }
                word |= (uint32_t)sidx << (8 * b);
            }
            segw[hr + 2 * q] = word;
            before += __shfl_sync(0xffffffffu, cinc, (threadIdx.x & 31 & ~3) | 3);
        }
        if (t == 0) nrec_s[row] = T.nrec[hr];
    }
}

// 0xFF in each byte of x equal to q, else 0
__device__ __forceinline__ uint32_t bytes_equal(uint32_t x, uint32_t q) {
    const uint32_t y = x ^ (q * 0x01010101u);
    const uint32_t nz = ((y & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | y;   // bit 7 set in non-zero bytes
    return prmt(~nz & 0x80808080u, 0u, 0xBA98u);                    // replicate bit 7 over the byte
}

template <bool WIDE>
__global__ void __launch_bounds__(AM_THREADS, 1)
k_attention_mma(const int8_t *__restrict__ qkv, int ldq, const int8_t *__restrict__ kv_g,
                const int *__restrict__ chunk_row0, const int *__restrict__ chunk_len, int n_heads,
                const int32_t *__restrict__ score_mult, const int8_t *__restrict__ sink_key,
                const int16_t *__restrict__ rope_cos, const int16_t *__restrict__ rope_sin,
                const uint16_t *__restrict__ lut4k_g, int8_t *__restrict__ out, int ldo) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int task_ctr;
    const int c = blockIdx.x;
    const int r0 = chunk_row0[c], n = chunk_len[c];
    const int npad = (n + 31) & ~31;
    const int vt_ld = ((npad + 127) & ~127) + 32;   // 8 dims of a fragment land on distinct banks
    uint8_t *ks = smem;                              // [npad][64], dims permuted per thread quarter
    uint8_t *vt = ks + npad * 64;                    // [64][vt_ld], keys permuted per 32-key tile
    uint8_t *wsm = vt + 64 * vt_ld;
    const uint16_t *lut4k = lut4k_g;   // 8 KB, stays in L1
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    int *vst = reinterpret_cast<int *>(wsm + warp * AM_WARP_SMEM);   // [16][AM_ROW] folded state
    int *segbuf = vst + 16 * AM_ROW;                                 // [16][AM_ROW] segment sums
    uint32_t *rec_e = reinterpret_cast<uint32_t *>(segbuf + 16 * AM_ROW);  // [16][32]
    int *nrec_s = reinterpret_cast<int *>(rec_e + 16 * 32);          // [16]
    uint32_t *s_s = reinterpret_cast<uint32_t *>(nrec_s + 16);       // [16] final s (low 32 bits)

    // K row layout: bytes [16t' + 4k + b] = dim 16k + 4t' + b, so thread t reads its
    // four B words (dims 4t, 16+4t, 32+4t, 48+4t) as one 16-byte load.
    for (int i = tid; i < npad * 16; i += AM_THREADS) {
        const int key = i >> 4, wk = i & 15;   // source word: dims 4*wk .. 4*wk+3
        uint32_t v = 0, kw = 0;
        if (key < n) {
            const int8_t *src = kv_g + (size_t)(r0 + key) * 128;
            kw = *reinterpret_cast<const uint32_t *>(src + 4 * wk);
            v = *reinterpret_cast<const uint32_t *>(src + 64 + 4 * wk);
        }
        const int kq = wk >> 2, tq = wk & 3;   // dims 16*kq + 4*tq ..
        *reinterpret_cast<uint32_t *>(ks + key * 64 + 16 * tq + 4 * kq) = kw;
        // V^T: tile position of key: keys 4u..4u+3 -> 8u + 0..3, keys 16+4u.. -> 8u + 4..7
        const int kt = key & 31;
        const int pos = (key & ~31) + 8 * ((kt & 15) >> 2) + 4 * (kt >> 4) + (kt & 3);
#pragma unroll
        for (int b = 0; b < 4; b++) vt[(4 * wk + b) * vt_ld + pos] = (uint8_t)(v >> (8 * b));
    }
    if (tid == 0) task_ctr = 0;
    __syncthreads();

    const uint32_t c8 = 378194u << 8;   // ATTN_COEF_Q24 (attention.rs:14-19) << 8
    const int n_rb = (n + 15) >> 4;
    const int n_tasks = n_rb * n_heads;
    for (;;) {
        int task = 0;
        if (lane == 0) task = atomicAdd(&task_ctr, 1);
        task = __shfl_sync(0xffffffffu, task, 0);
        if (task >= n_tasks) break;
        const int rb = n_rb - 1 - task / n_heads;   // longest rows first
        const int h = task % n_heads;
        const int p0 = rb * 16;
        const int prow[2] = {p0 + g, p0 + g + 8};
        const int p_last = min(p0 + 15, n - 1);
        const bool full_rows = p0 + 15 < n;
        const int mult = score_mult[h];

        // Q fragments with RoPE (attention.rs:53-83); pairs (i, i+32) live in kk = 0 / 1
        uint32_t qa[2][4];
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            const int p = prow[hr];
            uint32_t raw[4] = {0, 0, 0, 0};   // dims 4t, 16+4t, 32+4t, 48+4t (+0..3)
            if (p < n) {
                const int8_t *qr = qkv + (size_t)(r0 + p) * ldq + h * 64;
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
                    if (p < n) { cs = rope_cos[p * kHalfDim + i]; sn = rope_sin[p * kHalfDim + i]; }
                    int xr = clamp127(sra_rne32(sra_rne32(x * cs - y * sn, 15), 1));
                    int yr = clamp127(sra_rne32(sra_rne32(x * sn + y * cs, 15), 1));
                    lo[k] |= (uint32_t)(uint8_t)xr << (8 * b);
                    hi[k] |= (uint32_t)(uint8_t)yr << (8 * b);
                }
            qa[0][hr] = lo[0];
            qa[0][hr + 2] = lo[1];
            qa[1][hr] = hi[0];
            qa[1][hr + 2] = hi[1];
        }

        // per-row running max and weight sums, replicated over the quad
        int m[2] = {INT32_MIN, INT32_MIN};
        unsigned long long s_state[2] = {0, 0};
        int sh[4] = {0, 0, 0, 0}, sl[4] = {0, 0, 0, 0};   // weight sums since the last fold
        if (sink_key != nullptr) {   // attention.rs:211-224
            int accs[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                uint32_t b0 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 4 * t);
                uint32_t b1 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 16 + 4 * t);
                mma_s8s8(accs, qa[kk], b0, b1);   // every B column is the sink key
            }
            m[0] = score_from_dot<true>(accs[0], mult);
            m[1] = score_from_dot<true>(accs[2], mult);
            s_state[0] = s_state[1] = 65535ull;
        }
        for (int i = lane; i < 16 * AM_ROW; i += 32) vst[i] = 0;
        int hiacc[8][4], loacc[8][4];
#pragma unroll
        for (int jd = 0; jd < 8; jd++)
#pragma unroll
            for (int k = 0; k < 4; k++) { hiacc[jd][k] = 0; loacc[jd][k] = 0; }

        for (int kb = 0; kb <= p_last; kb += 32) {
            // ---- S = Q K^T over 32 keys (permuted columns) ----
            int sacc[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0;
                const uint4 kw = *reinterpret_cast<const uint4 *>(ks + (kb + perm_key(8 * j + g)) * 64 + 16 * t);
                mma_s8s8(sacc[j], qa[0], kw.x, kw.y);
                mma_s8s8(sacc[j], qa[1], kw.z, kw.w);
            }
            uint2 bv[8];
#pragma unroll
            for (int jd = 0; jd < 8; jd++)
                bv[jd] = *reinterpret_cast<const uint2 *>(vt + (8 * jd + g) * vt_ld + kb + 8 * t);

            Tile T;
            if (!full_rows || kb + 31 > p0)
                tile_softmax<true, WIDE>(sacc, kb, prow, n, mult, t, lane, m, lut4k, c8, T);
            else
                tile_softmax<false, WIDE>(sacc, kb, prow, n, mult, t, lane, m, lut4k, c8, T);
            // full P fragments (u8 halves of the weights)
            uint32_t phi[4], plo[4];
#pragma unroll
            for (int hr = 0; hr < 2; hr++)
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const uint32_t *wq = &T.w[hr][4 * q];
                    const uint32_t x01 = prmt(wq[0], wq[1], 0x5140u);   // lo0 lo1 hi0 hi1
                    const uint32_t x23 = prmt(wq[2], wq[3], 0x5140u);
                    plo[hr + 2 * q] = prmt(x01, x23, 0x5410u);
                    phi[hr + 2 * q] = prmt(x01, x23, 0x7632u);
                }
            const int maxrec = (int)__reduce_max_sync(0xffffffffu, (unsigned)max(T.nrec[0], T.nrec[1]));
            uint32_t segw[4] = {0, 0, 0, 0};
            if (maxrec > 0) {
                tile_segments(T, t, g, rec_e, nrec_s, segw);
                __syncwarp();
            }
            for (int pass = 0; pass <= maxrec; pass++) {
                if (pass > 0) {
                    // rows with a pass-th record hand their segment sums to the warp
#pragma unroll
                    for (int hr = 0; hr < 2; hr++) {
                        if (T.nrec[hr] >= pass) {
                            const int row = g + 8 * hr;
                            const uint32_t f = rec_e[row * 32 + pass - 1];
                            const unsigned long long stot = s_state[hr] +
                                256ull * (uint32_t)sh[2 * hr] + (unsigned long long)(uint32_t)sl[2 * hr];
                            s_state[hr] = (f & 0x20000u) ? stot : (stot * (f & 0xFFFFu) + 0x8000ull) >> 16;
                            sh[2 * hr] = sh[2 * hr + 1] = sl[2 * hr] = sl[2 * hr + 1] = 0;
#pragma unroll
                            for (int jd = 0; jd < 8; jd++) {
                                int2 v2;
                                v2.x = (int)(((uint32_t)hiacc[jd][2 * hr] << 8) + (uint32_t)loacc[jd][2 * hr]);
                                v2.y = (int)(((uint32_t)hiacc[jd][2 * hr + 1] << 8) + (uint32_t)loacc[jd][2 * hr + 1]);
                                *reinterpret_cast<int2 *>(segbuf + row * AM_ROW + 8 * jd + 2 * t) = v2;
                                hiacc[jd][2 * hr] = hiacc[jd][2 * hr + 1] = 0;
                                loacc[jd][2 * hr] = loacc[jd][2 * hr + 1] = 0;
                            }
                        }
                    }
                    const uint32_t fold0 = __ballot_sync(0xffffffffu, t == 0 && T.nrec[0] >= pass);
                    const uint32_t fold1 = __ballot_sync(0xffffffffu, t == 0 && T.nrec[1] >= pass);
                    __syncwarp();
                    // the whole warp folds each such row, 2 dims per lane (attention.rs:252-263)
                    uint32_t rows = 0;
#pragma unroll
                    for (int k = 0; k < 8; k++) rows |= (((fold0 >> (4 * k)) & 1u) << k) | (((fold1 >> (4 * k)) & 1u) << (k + 8));
                    while (rows) {
                        const int row = __ffs(rows) - 1;
                        rows &= rows - 1;
                        const uint32_t f = rec_e[row * 32 + pass - 1];
                        const long long e = f & 0xFFFFu;
                        int2 sv = *reinterpret_cast<int2 *>(vst + row * AM_ROW + 2 * lane);
                        const int2 gv = *reinterpret_cast<const int2 *>(segbuf + row * AM_ROW + 2 * lane);
                        uint32_t x0 = (uint32_t)sv.x + (uint32_t)gv.x, x1 = (uint32_t)sv.y + (uint32_t)gv.y;
                        if (!(f & 0x20000u)) {
                            long long p0_ = (long long)(int)x0 * e, p1_ = (long long)(int)x1 * e;
                            p0_ += p0_ >= 0 ? (1ll << 15) : -(1ll << 15);
                            p1_ += p1_ >= 0 ? (1ll << 15) : -(1ll << 15);
                            x0 = (uint32_t)(int)(p0_ >> 16);
                            x1 = (uint32_t)(int)(p1_ >> 16);
                        }
                        sv.x = (int)x0;
                        sv.y = (int)x1;
                        *reinterpret_cast<int2 *>(vst + row * AM_ROW + 2 * lane) = sv;
                    }
                    __syncwarp();
                }
                // P fragments of this pass: bytes of entries in segment `pass`
                uint32_t ahi[4], alo[4];
                if (maxrec == 0) {
#pragma unroll
                    for (int a = 0; a < 4; a++) { ahi[a] = phi[a]; alo[a] = plo[a]; }
                } else {
#pragma unroll
                    for (int a = 0; a < 4; a++) {
                        const uint32_t mk = bytes_equal(segw[a], (uint32_t)pass);
                        ahi[a] = phi[a] & mk;
                        alo[a] = plo[a] & mk;
                    }
                }
                mma_u8s8(sh, ahi, 0x01010101u, 0x01010101u);   // weight sums (all-ones column)
                mma_u8s8(sl, alo, 0x01010101u, 0x01010101u);
#pragma unroll
                for (int jd = 0; jd < 8; jd++) {
                    mma_u8s8(hiacc[jd], ahi, bv[jd].x, bv[jd].y);
                    mma_u8s8(loacc[jd], alo, bv[jd].x, bv[jd].y);
                }
            }
        }

        // output: clamp(round_half_even(vacc / s)) (attention.rs:279-284)
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            const int row = g + 8 * hr;
#pragma unroll
            for (int jd = 0; jd < 8; jd++) {
                int2 v2;
                v2.x = (int)(((uint32_t)hiacc[jd][2 * hr] << 8) + (uint32_t)loacc[jd][2 * hr]);
                v2.y = (int)(((uint32_t)hiacc[jd][2 * hr + 1] << 8) + (uint32_t)loacc[jd][2 * hr + 1]);
                *reinterpret_cast<int2 *>(segbuf + row * AM_ROW + 8 * jd + 2 * t) = v2;
            }
            if (t == 0) {
                const unsigned long long s = s_state[hr] + 256ull * (uint32_t)sh[2 * hr] +
                                             (unsigned long long)(uint32_t)sl[2 * hr];
                s_s[row] = s == 0 ? 1u : (uint32_t)min(s, 0xFFFFFFFFull);
                nrec_s[row] = s > 0xFFFFFFFFull;   // s beyond 32 bits: every quotient is 0
            }
        }
        __syncwarp();
        for (int row = 0; row < 16; row++) {
            const int p = p0 + row;
            if (p >= n) break;
            const int2 sv = *reinterpret_cast<const int2 *>(vst + row * AM_ROW + 2 * lane);
            const int2 gv = *reinterpret_cast<const int2 *>(segbuf + row * AM_ROW + 2 * lane);
            const unsigned long long den = nrec_s[row] ? 0x100000000ull : s_s[row];
            const int x0 = (int)((uint32_t)sv.x + (uint32_t)gv.x), x1 = (int)((uint32_t)sv.y + (uint32_t)gv.y);
            const uint16_t pk = (uint16_t)(uint8_t)clamp127(div_rne_s32_u64(x0, den)) |
                                ((uint16_t)(uint8_t)clamp127(div_rne_s32_u64(x1, den)) << 8);
            *reinterpret_cast<uint16_t *>(out + (size_t)(r0 + p) * ldo + h * 64 + 2 * lane) = pk;
        }
        __syncwarp();
    }
}

}  // namespace

size_t attention_mma_smem(int max_len) {
    const int npad = (max_len + 31) & ~31;
    const int vt_ld = ((npad + 127) & ~127) + 32;
    return (size_t)npad * 64 + (size_t)64 * vt_ld + (size_t)AM_WARPS * AM_WARP_SMEM;
}

bool attention_mma_fits(int max_len) { return max_len <= AM_MAX_KEYS; }

void attention_mma_init() {
    cudaFuncSetAttribute(k_attention_mma<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)attention_mma_smem(AM_MAX_KEYS));
    cudaFuncSetAttribute(k_attention_mma<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)attention_mma_smem(AM_MAX_KEYS));
}

void launch_attention_mma(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                          const int *chunk_len, int n_chunks, int max_len, int n_heads,
                          const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                          const int16_t *rope_sin, const uint16_t *lut4k, bool wide_mult, int8_t *out,
                          int ldo, cudaStream_t st) {
    if (n_chunks == 0) return;
    const size_t smem = attention_mma_smem(max_len);
    if (wide_mult)
        k_attention_mma<true><<<n_chunks, AM_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo);
    else
        k_attention_mma<false><<<n_chunks, AM_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut4k, out, ldo);
}

}  // namespace czg
