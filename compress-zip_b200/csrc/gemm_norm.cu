// gemm_norm.cu -- the O and down projections with the sandwich norm, the residual
// add and the next pre-norm fused into the GEMM epilogue, so the projection output
// never goes through HBM.
//
// Computes, per row (rust/src/model.rs:418-438 after the O projection, 455-475 after
// the down projection):
//   o   = requant(x . W^T)                        (linear.rs:12-31, model.rs:280-300)
//   y   = rmsnorm(o, post_w)                      (rmsnorm.rs:40-75)
//   res = res + y (int32 in the reference, never clamped; int16 here when exact)
//   xn  = rmsnorm(clamp_i8(res), next_w)          the next GEMM's input
// A norm needs the sum of squares of the whole row, so one CTA owns whole rows: the
// output width d is two tiles of d/2 columns (N = d/2 per tcgen05.mma), computed one
// after the other into the two TMEM accumulators.  Roles as in gemm_tc.cu: warp 0
// lane 0 TMA producer, warp 1 lane 0 MMA issuer, warps 2..17 epilogue (four per TMEM
// lane quadrant, one row per lane, each a quarter of the row's columns).  For the
// tile holding its quarter an epilogue warp requantises its TMEM columns (exact FP32
// form, common.cuh) into a shared-memory copy of the row block's int8 output and adds
// to the row's sum of squares, then releases the accumulator, so the next row
// block's MMAs overlap the norm phase.  The four warps of a quadrant combine their
// sums through shared memory at a named barrier; then each warp takes 8 of the
// quadrant's rows one at a time, its lanes across the row (coalesced like rows.cu),
// normalises, adds the residual (from HBM, or the embedding row for the first norm
// of the model), stores it back, clamps, and writes the next pre-norm's output.  Every mbarrier wait
// is bounded (kErrTimeout, as gemm_tc.cu).  No TMA load here uses cluster multicast.
#include "kernels.h"
#include "tc_common.cuh"

namespace czg {
namespace {

constexpr int GN_EPI = 16;                    // epilogue warps: four per TMEM lane quadrant
constexpr int GN_THREADS = 64 + 32 * GN_EPI;
constexpr int GN_STAGES = 3;

// modes of the residual (as rows.cu): read x_res and write it back; read the embedding
// row of tok_in and write x_res; read x_res and write nothing back (the model's last norm)
enum { kGnFromRes = 0, kGnFromEmbed = 1, kGnNoStore = 2 };

struct GnArgs {
    const int8_t *post_w, *next_w;   // [d] int8 norm weights
    const uint16_t *inv_tab;          // inv_rms_q15 by floor(sum_sq / d)
    const uint32_t *tok_in;           // kGnFromEmbed: embedding row of each row
    const int8_t *embed;
    void *x_res;                      // [M][d] residual (int16 or int32)
    int8_t *xn;                       // [M][d] next pre-norm output
    float mf, c2;                     // requantisation: mult / 2^shift, M1 - M1 * mult / 2^shift
    int clamp_a;                      // accumulator clamp bound (result stays within +-127)
};

template <int D>
struct GnCfg {
    static constexpr int BN = D / 2;                       // columns per tile, two tiles per row block
    static constexpr int Q = D / 4;                        // columns per epilogue warp
    static constexpr int TMEM_COLS = D <= 256 ? 256 : 512; // two accumulators of BN columns
    static constexpr int A_BYTES = TC_BM * TC_BK;
    static constexpr int B_BYTES = BN * TC_BK;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int PITCH = D + 16;                   // row pitch of the output copy (16-byte phases)
    static constexpr size_t SMEM = 1024 + (size_t)GN_STAGES * STAGE + (size_t)TC_BM * PITCH + 2 * D +
                                   3 * 4 * 4 * 32 * 4 + (2 * GN_STAGES + 6) * 8 + 16;
};

__device__ __forceinline__ void bar_quadrant(int q) {   // the 4 epilogue warps of lane quadrant q
    asm volatile("bar.sync %0, 128;" ::"r"(1 + q) : "memory");
}

// biased bits of the FP32 requantisation of an accumulator (gemm_tc.cu, rq_flt)
__device__ __forceinline__ int rq_bits(int acc, const GnArgs &a) {
    const int b = min(__viaddmax_s32(acc, (int)kM1Bits, (int)kM1Bits - a.clamp_a), (int)kM1Bits + a.clamp_a);
    return __float_as_int(__fmaf_rn(__int_as_float(b), a.mf, a.c2));
}

struct GnNorm {
    float mf, c;   // inv / 2^15, M1 - 384 inv
};
__device__ __forceinline__ GnNorm gn_norm(int sum_sq, const uint16_t *__restrict__ inv_tab, int d) {
    const int inv = __ldg(inv_tab + min((uint32_t)sum_sq / (uint32_t)d, (uint32_t)kInvTabEntries - 1u));
    return GnNorm{__int2float_rn(inv) * (1.0f / 32768.0f), __int2float_rn(12582912 - 384 * inv)};
}
// biased bits of clamp(rne(x * w * inv / 2^15), +-127) (rows.cu, norm_b)
__device__ __forceinline__ int gn_norm_b(int x, int w, const GnNorm &n) {
    const int yb = __float_as_int(__fmaf_rn(__int_as_float(x * w + (int)kM1Bits), n.mf, n.c));
    return min(max(yb, (int)kM1Bits - 127), (int)kM1Bits + 127);
}
// the same without the clamp: the biased bits, whose low 16 bits are the int16 y, since
// |y| <= 127 * 128 * 65535 / 2^15 < 2^15 (inv_tab entries are 16-bit)
__device__ __forceinline__ int gn_norm_f(int x, int w, const GnNorm &n) {
    return __float_as_int(__fmaf_rn(__int_as_float(x * w + (int)kM1Bits), n.mf, n.c));
}
// two such results as an int16 pair clamped to +-127
__device__ __forceinline__ uint32_t gn_pair127(int f0, int f1) {
    return __vmaxs2(__vmins2(__byte_perm(f0, f1, 0x5410), 0x007F007Fu), 0xFF81FF81u);
}
// byte b of w sign-extended: prmt's default mode copies byte b and replicates its sign
__device__ __forceinline__ int sx8(uint32_t w, int b) {
    uint32_t r;
    switch (b) {
        case 0: asm("prmt.b32 %0, %1, 0, 0x8880;" : "=r"(r) : "r"(w)); break;
        case 1: asm("prmt.b32 %0, %1, 0, 0x9991;" : "=r"(r) : "r"(w)); break;
        case 2: asm("prmt.b32 %0, %1, 0, 0xAAA2;" : "=r"(r) : "r"(w)); break;
        default: asm("prmt.b32 %0, %1, 0, 0xBBB3;" : "=r"(r) : "r"(w)); break;
    }
    return (int)r;
}
__device__ __forceinline__ uint32_t pk4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

__device__ __forceinline__ void store_res4(int16_t *p, const int (&r)[4]) {
    *reinterpret_cast<uint2 *>(p) = make_uint2(((uint32_t)r[0] & 0xFFFFu) | ((uint32_t)r[1] << 16),
                                               ((uint32_t)r[2] & 0xFFFFu) | ((uint32_t)r[3] << 16));
}
__device__ __forceinline__ void store_res4(int32_t *p, const int (&r)[4]) {
    *reinterpret_cast<int4 *>(p) = make_int4(r[0], r[1], r[2], r[3]);
}

// A row's residual words as loaded (int16 pairs, int32 quads, or embedding bytes),
// so a row can be loaded while the previous one is processed.
template <typename RT, int MODE>
struct GnRaw {
    using T = uint2;
};
template <int MODE>
struct GnRaw<int32_t, MODE> {
    using T = int4;
};
template <>
struct GnRaw<int16_t, kGnFromEmbed> {
    using T = uint32_t;
};
template <>
struct GnRaw<int32_t, kGnFromEmbed> {
    using T = uint32_t;
};
__device__ __forceinline__ void gn_unpack(uint2 u, int (&r)[4]) {
    r[0] = (int)(int16_t)(u.x & 0xFFFFu); r[1] = (int)(int16_t)(u.x >> 16);
    r[2] = (int)(int16_t)(u.y & 0xFFFFu); r[3] = (int)(int16_t)(u.y >> 16);
}
__device__ __forceinline__ void gn_unpack(int4 v, int (&r)[4]) {
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
}
__device__ __forceinline__ int sx8(uint32_t w, int b);
__device__ __forceinline__ void gn_unpack(uint32_t e, int (&r)[4]) {
#pragma unroll
    for (int b = 0; b < 4; b++) r[b] = sx8(e, b);
}
// the residual words of row `row` for this lane (zero beyond M or after an abort)
template <typename RT, int MODE, int NW>
__device__ __forceinline__ void gn_load_raw(const GnArgs &ga, int row, int M, bool alive, int lane,
                                            typename GnRaw<RT, MODE>::T (&w)[NW]) {
    using Raw = typename GnRaw<RT, MODE>::T;
    if (row < M && alive) {
        if constexpr (MODE == kGnFromEmbed) {
            const uint32_t *er = reinterpret_cast<const uint32_t *>(ga.embed + (size_t)ga.tok_in[row] * (NW * 128));
#pragma unroll
            for (int j = 0; j < NW; j++) w[j] = __ldg(er + lane + 32 * j);
        } else {
            const RT *xr = reinterpret_cast<const RT *>(ga.x_res) + (size_t)row * (NW * 128);
#pragma unroll
            for (int j = 0; j < NW; j++) w[j] = *reinterpret_cast<const Raw *>(xr + 4 * lane + 128 * j);
        }
    } else {
#pragma unroll
        for (int j = 0; j < NW; j++) w[j] = Raw{};
    }
}

template <int D, typename RT, int MODE>
__global__ void __launch_bounds__(GN_THREADS, 1)
k_gemm_norm(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int K,
            GnArgs ga, int *__restrict__ err) {
    using C = GnCfg<D>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *o_s = smem + GN_STAGES * C::STAGE;                 // [128][PITCH] int8 output, then clamp(res)
    int8_t *w_s = reinterpret_cast<int8_t *>(o_s + TC_BM * C::PITCH);   // post_w, next_w
    int *xs = reinterpret_cast<int *>(w_s + 2 * D);   // sums [4 quadrants][4 parts][32] (one phase used), then flags
    uint64_t *full = reinterpret_cast<uint64_t *>(xs + 3 * 4 * 4 * 32);
    uint64_t *empty = full + GN_STAGES;
    uint64_t *tfull = empty + GN_STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = K / TC_BK;
    const int n_blocks = (M + TC_BM - 1) / TC_BM;
    const int my_blocks = n_blocks > (int)blockIdx.x ? (n_blocks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_vt = 2 * my_blocks;   // tiles: (block, column half)

    for (int i = threadIdx.x; i < D; i += GN_THREADS) {   // model constants
        w_s[i] = ga.post_w[i];
        w_s[D + i] = ga.next_w[i];
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < GN_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], GN_EPI / 2);   // the 8 warps whose quarters lie in that half
        }
        mbar_init(drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {   // TMA producer
            int it = 0;
            bool ok = true;
            for (int v = 0; v < n_vt && ok; v++) {
                const int m0 = ((int)blockIdx.x + (v >> 1) * (int)gridDim.x) * TC_BM, n0 = (v & 1) * C::BN;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % GN_STAGES;
                    if (it >= GN_STAGES && !mbar_wait(&empty[s], ((it / GN_STAGES) - 1) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + s * C::STAGE;
                    mbar_expect_tx(&full[s], C::STAGE);
                    tma_load_2d(sa, &map_a, &full[s], kb * TC_BK, m0);
                    tma_load_2d(sa + C::A_BYTES, &map_b, &full[s], kb * TC_BK, n0);
                }
            }
            if (!ok) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
                for (int k = max(0, it - GN_STAGES); k < it; k++)
                    mbar_wait(&full[k % GN_STAGES], (k / GN_STAGES) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer: tile v into accumulator v & 1
            const uint32_t idesc = idesc_i8(TC_BM, C::BN);
            int it = 0;
            bool ok = true;
            for (int v = 0; v < n_vt && ok; v++) {
                const int b = v & 1;
                if (v >= 2 && !mbar_wait(&tempty[b], ((v >> 1) - 1) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dt = tmem + (uint32_t)(b * C::BN);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % GN_STAGES;
                    if (!mbar_wait(&full[s], (it / GN_STAGES) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = smem_addr(smem + s * C::STAGE);
                    const uint64_t ad = smem_desc_sw128(sa);
                    const uint64_t bd = smem_desc_sw128(sa + C::A_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; k++) mma_i8(dt, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&tfull[b]);
            }
            if (!ok) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
            }
            mma_commit(drain);
            mbar_wait(drain, 0, nullptr);
        }
    } else {   // epilogue: row 32q + lane of each block, columns [part * Q, (part + 1) * Q)
        const int q = warp & 3, part = (warp - 2) >> 2, half = part >> 1;
        const int c0 = part * C::Q;
        uint8_t *orow = o_s + (32 * q + lane) * C::PITCH;
        constexpr int NW = D / 128;   // words of 4 columns per lane in the norm phase
        int w1[NW][4], w2[NW][4];     // post and next norm weights of this lane's columns
#pragma unroll
        for (int j = 0; j < NW; j++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                w1[j][b] = w_s[4 * lane + 128 * j + b];
                w2[j][b] = w_s[D + 4 * lane + 128 * j + b];
            }
        int *xq = xs + (q * 4) * 32;   // slot (phase, part) of this quadrant: xq[(phase * 16 + part) * 32 + lane]
        int *fq = xs + 2 * 512 + (q * 4) * 32;   // go / stop flags of the quadrant's warps, by part
        bool alive = true;
        for (int blk = 0; blk < my_blocks && alive; blk++) {
            const int v = 2 * blk + half, b = half;
            const int m0_blk = ((int)blockIdx.x + blk * (int)gridDim.x) * TC_BM;
            // ---- requantise this warp's quarter into the row copy; sum of squares ----
            const bool got = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (v >> 1) & 1, &abort_flag));
            if (!got) {
                if (lane == 0) {
                    atomicOr(err, kErrTimeout);
                    abort_flag = 1;
                }
                alive = false;
            }
            int ss = 0;
            if (alive) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * C::BN + (part & 1) * C::Q);
#pragma unroll 1
                for (int ch = 0; ch < C::Q / 32; ch++) {
                    uint32_t x[32];
                    tmem_ld32(tbase + 32 * ch, x);
                    uint32_t w[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        w[j] = pk4(rq_bits((int)x[4 * j], ga), rq_bits((int)x[4 * j + 1], ga),
                                   rq_bits((int)x[4 * j + 2], ga), rq_bits((int)x[4 * j + 3], ga));
                        ss = __dp4a((int)w[j], (int)w[j], ss);
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(orow + c0 + 32 * ch);
                    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);   // the accumulator is free for the next block
            }
            // every warp of the quadrant takes part in its barriers, alive or not; the
            // decision to go on is the same for all four (an abort seen by any stops all)
            xq[(0 * 16 + part) * 32 + lane] = ss;
            fq[part * 32 + lane] = (alive && !abort_flag) ? 1 : 0;
            bar_quadrant(q);
            alive = fq[0 * 32 + lane] & fq[1 * 32 + lane] & fq[2 * 32 + lane] & fq[3 * 32 + lane];
            alive = __all_sync(0xffffffffu, alive);
            // ---- norm phase: this warp takes 8 of the quadrant's rows, one at a time, its
            // lanes across the row (word j of lane l = columns 4l + 128j .. +3, as rows.cu),
            // so the residual and output traffic is coalesced ----
            using Raw = typename GnRaw<RT, MODE>::T;
            Raw nxt[NW];   // the next row's residual words, loaded a row ahead
            gn_load_raw<RT, MODE, NW>(ga, m0_blk + 32 * q + 8 * part, M, alive, lane, nxt);
#pragma unroll 1
            for (int i = 0; i < 8; i++) {
                const int rl = 8 * part + i;   // row within the quadrant
                const int grow = m0_blk + 32 * q + rl;
                Raw cur[NW];
#pragma unroll
                for (int j = 0; j < NW; j++) cur[j] = nxt[j];
                if (i < 7) gn_load_raw<RT, MODE, NW>(ga, grow + 1, M, alive, lane, nxt);
                const int ss1 = xq[(0 * 16 + 0) * 32 + rl] + xq[(0 * 16 + 1) * 32 + rl] +
                                xq[(0 * 16 + 2) * 32 + rl] + xq[(0 * 16 + 3) * 32 + rl];
                const GnNorm n1 = gn_norm(ss1, ga.inv_tab, D);
                const uint8_t *srow = o_s + (32 * q + rl) * C::PITCH;
                RT *xr = reinterpret_cast<RT *>(ga.x_res) + (size_t)grow * D;
                const bool live = grow < M && alive;
                int8_t *xo = ga.xn + (size_t)grow * D;
                if constexpr (sizeof(RT) == 2 && D <= 384) {
                    // int16 residual: the adds and clamps on int16 pairs (vadd as a 16x2
                    // add-max against -32768, vmin / vmax), the clamped row as bytes for a
                    // dp4a sum of squares and the next norm (-8% at d = 384; at d = 512 the
                    // O projection's kernel measured 9% slower this way, so it keeps the
                    // per-element form)
                    uint32_t cb[NW];
                    int ss2 = 0;
#pragma unroll
                    for (int j = 0; j < NW; j++) {
                        const int col = 4 * lane + 128 * j;
                        const uint32_t ov = *reinterpret_cast<const uint32_t *>(srow + col);
                        uint32_t r01, r23;
                        if constexpr (MODE == kGnFromEmbed) {   // embedding bytes to int16 pairs (prmt
                            // with sign replication; __byte_perm would ignore the selectors' top bits)
                            asm("prmt.b32 %0, %1, 0, 0x9180;" : "=r"(r01) : "r"((uint32_t)cur[j]));
                            asm("prmt.b32 %0, %1, 0, 0xB3A2;" : "=r"(r23) : "r"((uint32_t)cur[j]));
                        } else {
                            r01 = cur[j].x;
                            r23 = cur[j].y;
                        }
                        const uint32_t y01 = gn_pair127(gn_norm_f(sx8(ov, 0), w1[j][0], n1), gn_norm_f(sx8(ov, 1), w1[j][1], n1));
                        const uint32_t y23 = gn_pair127(gn_norm_f(sx8(ov, 2), w1[j][2], n1), gn_norm_f(sx8(ov, 3), w1[j][3], n1));
                        r01 = (uint32_t)__viaddmax_s16x2((int)r01, (int)y01, (int)0x80008000u);   // exact: |res| < 2^15
                        r23 = (uint32_t)__viaddmax_s16x2((int)r23, (int)y23, (int)0x80008000u);
                        if (MODE != kGnNoStore && live) *reinterpret_cast<uint2 *>(xr + col) = make_uint2(r01, r23);
                        const uint32_t c01 = __vmaxs2(__vmins2(r01, 0x007F007Fu), 0xFF81FF81u);
                        const uint32_t c23 = __vmaxs2(__vmins2(r23, 0x007F007Fu), 0xFF81FF81u);
                        cb[j] = __byte_perm(c01, c23, 0x6420);
                        ss2 = __dp4a((int)cb[j], (int)cb[j], ss2);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ss2 += __shfl_xor_sync(0xffffffffu, ss2, o);
                    const GnNorm n2 = gn_norm(ss2, ga.inv_tab, D);
#pragma unroll
                    for (int j = 0; j < NW; j++) {
                        const uint32_t g01 = gn_pair127(gn_norm_f(sx8(cb[j], 0), w2[j][0], n2), gn_norm_f(sx8(cb[j], 1), w2[j][1], n2));
                        const uint32_t g23 = gn_pair127(gn_norm_f(sx8(cb[j], 2), w2[j][2], n2), gn_norm_f(sx8(cb[j], 3), w2[j][3], n2));
                        if (live) *reinterpret_cast<uint32_t *>(xo + 4 * lane + 128 * j) = __byte_perm(g01, g23, 0x6420);
                    }
                    continue;
                }
                int cr[NW][4];
                int ss2 = 0;
#pragma unroll
                for (int j = 0; j < NW; j++) {
                    const int col = 4 * lane + 128 * j;
                    const uint32_t ov = *reinterpret_cast<const uint32_t *>(srow + col);
                    int res[4];
                    gn_unpack(cur[j], res);
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const int y = gn_norm_b(sx8(ov, b), w1[j][b], n1);
                        res[b] = (int)((uint32_t)res[b] + (uint32_t)y - kM1Bits);
                        cr[j][b] = min(max(res[b], -127), 127);
                        ss2 += cr[j][b] * cr[j][b];
                    }
                    if (MODE != kGnNoStore && live) store_res4(xr + col, res);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss2 += __shfl_xor_sync(0xffffffffu, ss2, o);
                const GnNorm n2 = gn_norm(ss2, ga.inv_tab, D);
#pragma unroll
                for (int j = 0; j < NW; j++) {
                    const uint32_t yw = pk4(gn_norm_b(cr[j][0], w2[j][0], n2), gn_norm_b(cr[j][1], w2[j][1], n2),
                                            gn_norm_b(cr[j][2], w2[j][2], n2), gn_norm_b(cr[j][3], w2[j][3], n2));
                    if (live) *reinterpret_cast<uint32_t *>(xo + 4 * lane + 128 * j) = yw;
                }
            }
            // the exchange slots and the row copy are reused by the next block
            bar_quadrant(q);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
}

template <int D, typename RT>
void set_attr_d() {
    cudaFuncSetAttribute(k_gemm_norm<D, RT, kGnFromRes>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)GnCfg<D>::SMEM);
    cudaFuncSetAttribute(k_gemm_norm<D, RT, kGnFromEmbed>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)GnCfg<D>::SMEM);
    cudaFuncSetAttribute(k_gemm_norm<D, RT, kGnNoStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)GnCfg<D>::SMEM);
}

template <int D, typename RT>
void launch_d(const CUtensorMap &ma, const CUtensorMap &mb, int M, int K, int mode, const GnArgs &ga, int *err,
              cudaStream_t st) {
    const int n_blocks = (M + TC_BM - 1) / TC_BM;
    const int grid = n_blocks < sm_count() ? n_blocks : sm_count();
    if (mode == kGnFromEmbed)
        launch_k(k_gemm_norm<D, RT, kGnFromEmbed>, grid, GN_THREADS, GnCfg<D>::SMEM, st, ma, mb, M, K, ga, err);
    else if (mode == kGnNoStore)
        launch_k(k_gemm_norm<D, RT, kGnNoStore>, grid, GN_THREADS, GnCfg<D>::SMEM, st, ma, mb, M, K, ga, err);
    else
        launch_k(k_gemm_norm<D, RT, kGnFromRes>, grid, GN_THREADS, GnCfg<D>::SMEM, st, ma, mb, M, K, ga, err);
}

}  // namespace

void gemm_norm_init() {
    set_attr_d<256, int16_t>();
    set_attr_d<384, int16_t>();
    set_attr_d<512, int16_t>();
    set_attr_d<256, int32_t>();
    set_attr_d<384, int32_t>();
    set_attr_d<512, int32_t>();
}

bool gemm_norm_supported(int d) { return d == 256 || d == 384 || d == 512; }

bool launch_gemm_norm(const TcMatrix &A, const TcMatrix &B, int M, int d, int K, int mult, int shift,
                      const int8_t *post_w, const int8_t *next_w, const uint16_t *inv_tab, const uint32_t *tok_in,
                      const int8_t *embed, bool store_res, void *x_res, bool res16, int8_t *xn, int *err,
                      cudaStream_t st) {
    if (M <= 0) return true;
    GnArgs ga{};
    if (!gemm_norm_supported(d) || B.box_rows != d / 2 || A.box_rows != TC_BM || K % TC_BK != 0 ||
        (long long)K * 16256 >= (1ll << 29) || !requant_fp32(mult, shift, &ga.mf, &ga.c2, &ga.clamp_a))
        return false;
    ga.post_w = post_w;
    ga.next_w = next_w;
    ga.inv_tab = inv_tab;
    ga.tok_in = tok_in;
    ga.embed = embed;
    ga.x_res = x_res;
    ga.xn = xn;
    const int mode = embed != nullptr ? kGnFromEmbed : (store_res ? kGnFromRes : kGnNoStore);
    const CUtensorMap &ma = *reinterpret_cast<const CUtensorMap *>(A.map);
    const CUtensorMap &mb = *reinterpret_cast<const CUtensorMap *>(B.map);
    switch (d) {
        case 256:
            res16 ? launch_d<256, int16_t>(ma, mb, M, K, mode, ga, err, st) : launch_d<256, int32_t>(ma, mb, M, K, mode, ga, err, st);
            break;
        case 384:
            res16 ? launch_d<384, int16_t>(ma, mb, M, K, mode, ga, err, st) : launch_d<384, int32_t>(ma, mb, M, K, mode, ga, err, st);
            break;
        default:
            res16 ? launch_d<512, int16_t>(ma, mb, M, K, mode, ga, err, st) : launch_d<512, int32_t>(ma, mb, M, K, mode, ga, err, st);
            break;
    }
    return true;
}

}  // namespace czg
