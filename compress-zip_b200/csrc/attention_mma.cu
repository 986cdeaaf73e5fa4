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
// of segment q (segment = run of keys between records), and before pass q every
// row with a q-th record folds its state exactly as the reference rescales at
// that key: state = R(state + 256*Hi + Lo, e), s = ((s + seg_sum) * e + 2^15) >> 16.
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int AM_THREADS = 256;
constexpr int AM_WARPS = AM_THREADS / 32;
constexpr int AM_MAX_KEYS = 1024;

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

// exp_q16 with the attention coefficient via a 4096-entry table indexed by
// t256 (entries for t256 >= 4096 are all 1, whatever the exp2 LUT holds).
// t256 = floor((neg * coef + 2^23) / 2^24) = hi + (lo >= 2^31) of neg * (coef << 8).
__device__ __forceinline__ uint32_t exp_attn(int diff, const uint16_t *lut4k, uint32_t c8) {
    if (diff >= 0) return 65535u;
    uint32_t neg = 0u - (uint32_t)diff;
    uint32_t t = __umulhi(neg, c8) + ((neg * c8) >> 31);
    return t < 4096u ? (uint32_t)lut4k[t] : 1u;
}

__device__ __forceinline__ int score_from_dot(int dot, int mult) {
    return sra_rne64_to32((long long)sra_rne32(dot, 2) * (long long)mult, 15);
}

// quad (4 lanes with equal lane>>2) helpers
__device__ __forceinline__ uint32_t quad_or(uint32_t v) {
    v |= __shfl_xor_sync(0xffffffffu, v, 1);
    v |= __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}
__device__ __forceinline__ uint32_t quad_sum(uint32_t v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// key of accumulator column n = 8j + 2t + e in the QK product (and of B row n = 8j + g)
__device__ __forceinline__ int perm_key(int n) {
    int j = n >> 3, r = n & 7;
    return 16 * (j >> 1) + 4 * (r >> 1) + 2 * (j & 1) + (r & 1);
}

// K rows: 64 bytes, 16-byte chunks XOR-swizzled by (key >> 2) & 3
__device__ __forceinline__ uint32_t k_word(const uint8_t *ks, int key, int dim) {
    int chunk = (dim >> 4) ^ ((key >> 2) & 3);
    return *reinterpret_cast<const uint32_t *>(ks + key * 64 + chunk * 16 + (dim & 15));
}

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
    const int vt_ld = npad + 16;   // V^T row stride: 16-byte pad spreads the 8 dims of a fragment over banks
    uint8_t *ks = smem;                                   // [npad][64] swizzled
    uint8_t *vt = smem + npad * 64;                       // [64][vt_ld]
    uint16_t *lut4k = reinterpret_cast<uint16_t *>(vt + 64 * vt_ld);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;

    for (int i = tid; i < 4096 / 8; i += AM_THREADS)
        reinterpret_cast<uint4 *>(lut4k)[i] = reinterpret_cast<const uint4 *>(lut4k_g)[i];
    // K (rotated) rows -> swizzled smem; V -> transposed smem.  Rows >= n are zero.
    for (int i = tid; i < npad * 4; i += AM_THREADS) {
        int key = i >> 2, ch = i & 3;
        uint4 kw = make_uint4(0, 0, 0, 0);
        if (key < n) kw = *reinterpret_cast<const uint4 *>(kv_g + (size_t)(r0 + key) * 128 + ch * 16);
        *reinterpret_cast<uint4 *>(ks + key * 64 + ((ch ^ ((key >> 2) & 3)) * 16)) = kw;
    }
    for (int i = tid; i < npad * 16; i += AM_THREADS) {
        int key = i >> 4, q4 = i & 15;   // dims 4*q4 .. 4*q4+3 of key
        uint32_t v = 0;
        if (key < n) v = *reinterpret_cast<const uint32_t *>(kv_g + (size_t)(r0 + key) * 128 + 64 + 4 * q4);
#pragma unroll
        for (int b = 0; b < 4; b++) vt[(4 * q4 + b) * vt_ld + key] = (uint8_t)(v >> (8 * b));
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
            // kk = 0: dims 0..31 -> a0/a1 = dims 4t.., a2/a3 = dims 16+4t..; kk = 1: +32
            qa[0][hr] = lo[0];
            qa[0][hr + 2] = lo[1];
            qa[1][hr] = hi[0];
            qa[1][hr + 2] = hi[1];
        }

        // per-row state, replicated over the quad
        int m[2] = {INT32_MIN, INT32_MIN};
        unsigned long long s_state[2] = {0, 0};
        uint32_t s_seg[2] = {0, 0};
        if (sink_key != nullptr) {   // attention.rs:211-224
            // sink score of each row: dot(q_rot, sink) via the same fragments
            int accs[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                uint32_t b0 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 4 * t);
                uint32_t b1 = *reinterpret_cast<const uint32_t *>(sink_key + 32 * kk + 16 + 4 * t);
                mma_s8s8(accs, qa[kk], b0, b1);   // every B column is the sink key
            }
            m[0] = score_from_dot(accs[0], mult);
            m[1] = score_from_dot(accs[2], mult);
            s_state[0] = s_state[1] = 65535ull;
        }
        uint32_t vst[2][8][2];
        int hiacc[8][4], loacc[8][4];
#pragma unroll
        for (int jd = 0; jd < 8; jd++)
#pragma unroll
            for (int k = 0; k < 4; k++) { hiacc[jd][k] = 0; loacc[jd][k] = 0; }
#pragma unroll
        for (int hr = 0; hr < 2; hr++)
#pragma unroll
            for (int jd = 0; jd < 8; jd++) { vst[hr][jd][0] = 0; vst[hr][jd][1] = 0; }

        for (int kb = 0; kb <= p_last; kb += 32) {
            // ---- S = Q K^T over 32 keys (permuted columns) ----
            int sacc[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int k = 0; k < 4; k++) sacc[j][k] = 0;
#pragma unroll
            for (int kk = 0; kk < 2; kk++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int key = kb + perm_key(8 * j + g);
                    uint32_t b0 = k_word(ks, key, 32 * kk + 4 * t);
                    uint32_t b1 = k_word(ks, key, 32 * kk + 16 + 4 * t);
                    mma_s8s8(sacc[j], qa[kk], b0, b1);
                }
            // V^T fragments for this tile (reused by every pass)
            uint32_t bv[8][2];
#pragma unroll
            for (int jd = 0; jd < 8; jd++) {
                const uint8_t *row = vt + (8 * jd + g) * vt_ld + kb + 4 * t;
                bv[jd][0] = *reinterpret_cast<const uint32_t *>(row);
                bv[jd][1] = *reinterpret_cast<const uint32_t *>(row + 16);
            }

            // ---- scores, prefix max, records, weights (entry i: key kb + 16*(i>>2) + 4t + (i&3)) ----
            uint32_t w[2][8], ef[2][8];
            uint32_t recmask[2] = {0, 0};
            int seg[2][8];
            int nrec[2];
#pragma unroll
            for (int hr = 0; hr < 2; hr++) {
                int sc[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int q = i >> 2, b = i & 3;
                    const int j = 2 * q + (b >> 1), e = b & 1;
                    const int key = kb + 16 * q + 4 * t + b;
                    const bool valid = key <= prow[hr] && prow[hr] < n;
                    sc[i] = valid ? score_from_dot(sacc[j][2 * hr + e], mult) : INT32_MIN;
                }
                int run = m[hr];
                int cnt_before = 0;
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
                    int excl = __shfl_up_sync(0xffffffffu, inc, 1, 4);
                    const int base = t == 0 ? run : max(run, excl);
                    int prevmax = base;
                    int lrec = 0;
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int i = 4 * q + b;
                        const int key = kb + 16 * q + 4 * t + b;
                        const bool valid = key <= prow[hr] && prow[hr] < n;
                        const int pm = max(base, L[b]);
                        const bool rec = valid && sc[i] > prevmax;
                        w[hr][i] = valid ? exp_attn((int)((uint32_t)sc[i] - (uint32_t)pm), lut4k, c8) : 0u;
                        // record flag 0x10000 | rescale factor, or 0x20000 when the previous max
                        // is still INT32_MIN: the reference then keeps its sums unscaled
                        ef[hr][i] = !rec ? 0u
                                    : prevmax == INT32_MIN
                                        ? 0x20000u
                                        : 0x10000u | exp_attn((int)((uint32_t)prevmax - (uint32_t)sc[i]), lut4k, c8);
                        if (rec) { recmask[hr] |= 1u << i; lrec++; }
                        prevmax = pm;
                    }
                    // segment index of each entry: records at or before it in this tile
                    int cinc = lrec;
                    int cu = __shfl_up_sync(0xffffffffu, cinc, 1, 4);
                    if (t >= 1) cinc += cu;
                    cu = __shfl_up_sync(0xffffffffu, cinc, 2, 4);
                    if (t >= 2) cinc += cu;
                    int cex = __shfl_up_sync(0xffffffffu, cinc, 1, 4);
                    int sidx = cnt_before + (t == 0 ? 0 : cex);
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int i = 4 * q + b;
                        if ((recmask[hr] >> i) & 1u) sidx++;
                        seg[hr][i] = sidx;
                    }
                    cnt_before += __shfl_sync(0xffffffffu, cinc, (lane & ~3) | 3);
                    run = max(run, __shfl_sync(0xffffffffu, inc, (lane & ~3) | 3));
                }
                m[hr] = run;
                nrec[hr] = cnt_before;
            }
            const int passes = 1 + __reduce_max_sync(0xffffffffu, (unsigned)max(nrec[0], nrec[1]));

            for (int pass = 0; pass < passes; pass++) {
                if (pass > 0) {
#pragma unroll
                    for (int hr = 0; hr < 2; hr++) {
                        uint32_t cand = 0;
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            if (((recmask[hr] >> i) & 1u) && seg[hr][i] == pass) cand = ef[hr][i];
                        cand = quad_or(cand);
                        if (cand) {   // fold exactly as the reference rescales (attention.rs:248-263)
                            const bool scale = (cand & 0x20000u) == 0;
                            const unsigned long long e = cand & 0xFFFFu;
                            const unsigned long long stot = s_state[hr] + s_seg[hr];
                            s_state[hr] = scale ? (stot * e + 0x8000ull) >> 16 : stot;
                            s_seg[hr] = 0;
#pragma unroll
                            for (int jd = 0; jd < 8; jd++)
#pragma unroll
                                for (int k = 0; k < 2; k++) {
                                    uint32_t x = vst[hr][jd][k] + ((uint32_t)hiacc[jd][2 * hr + k] << 8) +
                                                 (uint32_t)loacc[jd][2 * hr + k];
                                    if (scale) {
                                        long long pr = (long long)(int)x * (long long)e;
                                        pr += pr >= 0 ? (1ll << 15) : -(1ll << 15);
                                        x = (uint32_t)(int)(pr >> 16);
                                    }
                                    vst[hr][jd][k] = x;
                                    hiacc[jd][2 * hr + k] = 0;
                                    loacc[jd][2 * hr + k] = 0;
                                }
                        }
                    }
                }
                // P fragments of this pass: weights of keys in segment `pass`
                uint32_t ahi[4], alo[4];
#pragma unroll
                for (int hr = 0; hr < 2; hr++) {
                    uint32_t ssum = 0;
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        uint32_t ph = 0, pl = 0;
#pragma unroll
                        for (int b = 0; b < 4; b++) {
                            const int i = 4 * q + b;
                            const uint32_t wv = seg[hr][i] == pass ? w[hr][i] : 0u;
                            ssum += wv;
                            pl |= (wv & 0xFFu) << (8 * b);
                            ph |= (wv >> 8) << (8 * b);
                        }
                        alo[hr + 2 * q] = pl;
                        ahi[hr + 2 * q] = ph;
                    }
                    s_seg[hr] += quad_sum(ssum);
                }
#pragma unroll
                for (int jd = 0; jd < 8; jd++) {
                    mma_u8s8(hiacc[jd], ahi, bv[jd][0], bv[jd][1]);
                    mma_u8s8(loacc[jd], alo, bv[jd][0], bv[jd][1]);
                }
            }
        }

        // output: clamp(round_half_even(vacc / s)) (attention.rs:279-284)
#pragma unroll
        for (int hr = 0; hr < 2; hr++) {
            const int p = prow[hr];
            if (p >= n) continue;
            const unsigned long long s = s_state[hr] + s_seg[hr];
            const unsigned long long den = s == 0 ? 1ull : s;
            int8_t *o = out + (size_t)(r0 + p) * ldo + h * 64 + 2 * t;
#pragma unroll
            for (int jd = 0; jd < 8; jd++) {
                uint32_t x0 = vst[hr][jd][0] + ((uint32_t)hiacc[jd][2 * hr] << 8) + (uint32_t)loacc[jd][2 * hr];
                uint32_t x1 = vst[hr][jd][1] + ((uint32_t)hiacc[jd][2 * hr + 1] << 8) + (uint32_t)loacc[jd][2 * hr + 1];
                uint16_t pk = (uint16_t)(uint8_t)clamp127(div_rne_s32_u64((int)x0, den)) |
                              ((uint16_t)(uint8_t)clamp127(div_rne_s32_u64((int)x1, den)) << 8);
                *reinterpret_cast<uint16_t *>(o + 8 * jd) = pk;
            }
        }
    }
}

}  // namespace

size_t attention_mma_smem(int max_len) {
    int npad = (max_len + 31) & ~31;
    return (size_t)npad * 64 + (size_t)64 * (npad + 16) + 4096 * 2;
}

bool attention_mma_fits(int max_len) { return max_len <= AM_MAX_KEYS; }

void attention_mma_init() {
    cudaFuncSetAttribute(k_attention_mma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)attention_mma_smem(AM_MAX_KEYS));
}

void launch_attention_mma(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                          const int *chunk_len, int n_chunks, int max_len, int n_heads,
                          const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                          const int16_t *rope_sin, const uint16_t *lut4k, int8_t *out, int ldo,
                          cudaStream_t st) {
    if (n_chunks == 0) return;
    k_attention_mma<<<n_chunks, AM_THREADS, attention_mma_smem(max_len), st>>>(
        qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin, lut4k,
        out, ldo);
}

}  // namespace czg
