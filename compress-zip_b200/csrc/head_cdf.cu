// head_cdf.cu -- the LM head GEMM and the coder interval of each row's symbol in
// one persistent tcgen05 kernel, so the int32 logits never leave the chip.
//
// Same result as the head projection (rust/src/linear.rs:12-31 on the final-norm
// output) followed by build_cumfreqs (rust/src/softmax_cdf.rs:85-139) reduced to
// (cum[sym-1], cum[sym]) as k_cdf_lohi_reg computes it.  The CDF needs the row
// maximum before any weight and the weight sum before any frequency, so every
// 128-row block of logits is produced three times by the tensor cores (the head
// GEMM is 2 x V x d MAC per row, cheap next to a round trip of 4 V bytes per row
// through HBM):
//   pass 0: row maximum, maximum below the symbol, the symbol's logit;
//   pass 1: S = sum of exp_q16(logit - max) (table lookups);
//   pass 2: frequencies 1 + floor(e * (T - V) / S), summed over the whole row and
//           below the symbol, and the symbol's own.
// Roles as in gemm_tc.cu: warp 0 lane 0 TMA producer (A = 128 rows of the
// final-norm output, B = 256 rows of the head weight per 128-byte K block),
// warp 1 lane 0 MMA issuer into two TMEM accumulators of 256 columns, warps
// 2..17 epilogue: warp w reads TMEM lanes 32*(w%4).. (one row per lane), the
// HC_W warps of a quadrant each 256/HC_W of a tile's columns; at the end of a
// pass they combine their partial row values through shared memory, in step
// through a per-quadrant mbarrier.  Every wait is bounded (kErrTimeout, as
// gemm_tc.cu).  The epilogue (about 34 instructions per logit over the three
// passes) is the limit, not the tensor pipe (26% busy) or L2 (25%).
// Needs V % 256 == 0, K % 128 == 0, lut4k[0] == 65535, |logit| < 2^30, coef < 2^23.
// No TMA load here uses cluster multicast.
#include "kernels.h"
#include "tc_common.cuh"

namespace czg {
namespace {

constexpr int HC_BN = 256;
constexpr int HC_STAGES = 3;
constexpr int HC_W = 4;                  // epilogue warps per TMEM lane quadrant
constexpr int HC_EPI = 4 * HC_W;
constexpr int HC_THREADS = 64 + 32 * HC_EPI;
constexpr int HC_COLS = HC_BN / HC_W;    // tile columns per epilogue warp
constexpr int HC_LUT = 4104;
constexpr int HC_A = TC_BM * TC_BK;
constexpr int HC_B = HC_BN * TC_BK;
constexpr int HC_STAGE = HC_A + HC_B;
constexpr int HC_XCHG_WORDS = 4 * 3 * HC_W * 32 * 4;   // [quadrant][pass][warp][lane][4]
constexpr int HC_BARS = 2 * HC_STAGES + 5 + 12;
constexpr size_t HC_SMEM = 1024 + (size_t)HC_STAGES * HC_STAGE + HC_LUT * 2 + (size_t)HC_XCHG_WORDS * 4 +
                           (size_t)HC_BARS * 8 + 16;

// exp_q16 of (x - row max) by table: t256 = floor(((max - x) * coef + 2^23) / 2^24) is the
// high word of krow - x * (coef << 8), krow = max * (coef << 8) + 2^31 (one 64-bit product;
// coef < 2^23 and |x| < 2^30 keep it inside int64 and the word non-negative).
__device__ __forceinline__ uint32_t weight_of(long long krow, int x, const uint16_t *lut, int nc8) {
    return lut[min((uint32_t)(((long long)x * nc8 + krow) >> 32), 4096u)];
}

__global__ void __launch_bounds__(HC_THREADS, 1)
k_head_cdf(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int V,
           int K, const uint32_t *__restrict__ sym, const uint16_t *__restrict__ lut4k_g, uint32_t c8,
           uint32_t total, uint2 *__restrict__ lohi, int *__restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint16_t *lut = reinterpret_cast<uint16_t *>(smem + HC_STAGES * HC_STAGE);
    uint32_t *xchg = reinterpret_cast<uint32_t *>(lut + HC_LUT);
    uint64_t *full = reinterpret_cast<uint64_t *>(xchg + HC_XCHG_WORDS);
    uint64_t *empty = full + HC_STAGES;
    uint64_t *tfull = empty + HC_STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint64_t *xbar = drain + 1;   // [quadrant][pass]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xbar + 12);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = K / TC_BK;
    const int NT = V / HC_BN;
    const int per_mb = 3 * NT;   // virtual tiles per 128-row block: 3 passes x NT column tiles
    const int n_mb = (M + TC_BM - 1) / TC_BM;
    const int my_mb = n_mb > (int)blockIdx.x ? (n_mb - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_vt = my_mb * per_mb;

    for (int i = threadIdx.x; i < HC_LUT; i += HC_THREADS) lut[i] = lut4k_g[i];
    if (threadIdx.x == 0) {
        for (int s = 0; s < HC_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], HC_EPI);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < 12; i++) mbar_init(&xbar[i], HC_W);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(2 * HC_BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {   // TMA producer
            int it = 0;
            bool ok = true;
            for (int v = 0; v < n_vt && ok; v++) {
                const int m0 = ((int)blockIdx.x + (v / per_mb) * (int)gridDim.x) * TC_BM;
                const int n0 = ((v % per_mb) % NT) * HC_BN;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % HC_STAGES;
                    if (it >= HC_STAGES && !mbar_wait(&empty[s], ((it / HC_STAGES) - 1) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + s * HC_STAGE;
                    mbar_expect_tx(&full[s], HC_STAGE);
                    tma_load_2d(sa, &map_a, &full[s], kb * TC_BK, m0);
                    tma_load_2d(sa + HC_A, &map_b, &full[s], kb * TC_BK, n0);
                }
            }
            if (!ok) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
                for (int k = max(0, it - HC_STAGES); k < it; k++) mbar_wait(&full[k % HC_STAGES], (k / HC_STAGES) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            const uint32_t idesc = idesc_i8(TC_BM, HC_BN);
            int it = 0;
            bool ok = true;
            for (int v = 0; v < n_vt && ok; v++) {
                const int b = v & 1;
                if (v >= 2 && !mbar_wait(&tempty[b], ((v >> 1) - 1) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dt = tmem + (uint32_t)(b * HC_BN);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % HC_STAGES;
                    if (!mbar_wait(&full[s], (it / HC_STAGES) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = smem_addr(smem + s * HC_STAGE);
                    const uint64_t ad = smem_desc_sw128(sa);
                    const uint64_t bd = smem_desc_sw128(sa + HC_A);
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
    } else {   // epilogue: one row per lane
        const int q = warp & 3, h = (warp - 2) >> 2;
        const uint32_t R = total - (uint32_t)V;
        const int nc8 = -(int)c8;
        long long krow = 0;
        int mx = INT32_MIN, mb = INT32_MIN, xs = INT32_MIN;
        uint32_t S = 0, f_all = 0, f_below = 0, f_sym = 0, sy = 0;
        FreqDiv fd{};
        int row = 0;
        for (int v = 0; v < n_vt; v++) {
            const int mbi = v / per_mb, lv = v % per_mb;
            const int pass = lv / NT, n = lv % NT, b = v & 1;
            if (lv == 0) {   // a new block of rows
                row = ((int)blockIdx.x + mbi * (int)gridDim.x) * TC_BM + 32 * q + lane;
                sy = row < M ? sym[row] : 0xFFFFFFFFu;
                mx = mb = xs = INT32_MIN;
                S = f_all = f_below = f_sym = 0;
            }
            const bool got = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (v >> 1) & 1, &abort_flag));
            if (!got) {
                if (lane == 0) {
                    atomicOr(err, kErrTimeout);
                    abort_flag = 1;
                }
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * HC_BN + h * HC_COLS);
#pragma unroll 1
            for (int ch = 0; ch < HC_COLS / 32; ch++) {
                uint32_t x[32];
                tmem_ld32(tbase + 32 * ch, x);
                const uint32_t c0 = (uint32_t)(n * HC_BN + h * HC_COLS + 32 * ch);
                const bool whole_below = c0 + 32 <= sy, holds_sym = c0 <= sy && sy < c0 + 32;
                if (pass == 0) {
                    int cm = (int)x[0];
#pragma unroll
                    for (int k = 1; k < 32; k++) cm = max(cm, (int)x[k]);
                    mx = max(mx, cm);
                    if (whole_below) mb = max(mb, cm);
                    if (holds_sym) {
#pragma unroll
                        for (int k = 0; k < 32; k++) {
                            if (c0 + k < sy) mb = max(mb, (int)x[k]);
                            if (c0 + k == sy) xs = (int)x[k];
                        }
                    }
                } else if (pass == 1) {
#pragma unroll
                    for (int k = 0; k < 32; k++) S += weight_of(krow, (int)x[k], lut, nc8);
                } else if (!holds_sym) {
                    uint32_t fs = 0;
#pragma unroll
                    for (int k = 0; k < 32; k++) fs += freq_of(weight_of(krow, (int)x[k], lut, nc8), fd);
                    f_all += fs;
                    if (whole_below) f_below += fs;
                } else {
#pragma unroll
                    for (int k = 0; k < 32; k++) {
                        const uint32_t f = freq_of(weight_of(krow, (int)x[k], lut, nc8), fd);
                        f_all += f;
                        if (c0 + k < sy) f_below += f;
                        if (c0 + k == sy) f_sym = f;
                    }
                }
            }
            // the accumulator is free for the tile after next
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
            if (n != NT - 1) continue;
            // end of a pass: combine the row's partial values of the quadrant's warps
            uint32_t *mine = xchg + ((((q * 3 + pass) * HC_W) + h) * 32 + lane) * 4;
            if (pass == 0) { mine[0] = (uint32_t)mx; mine[1] = (uint32_t)mb; mine[2] = (uint32_t)xs; }
            else if (pass == 1) { mine[0] = S; }
            else { mine[0] = f_all; mine[1] = f_below; mine[2] = f_sym; }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xbar[q * 3 + pass]);
            if (!__all_sync(0xffffffffu, mbar_wait(&xbar[q * 3 + pass], mbi & 1, &abort_flag))) {
                if (lane == 0) {
                    atomicOr(err, kErrTimeout);
                    abort_flag = 1;
                }
                break;
            }
            uint32_t a0 = 0, a1 = 0, a2 = 0;
            int m0v = INT32_MIN, m1v = INT32_MIN, m2v = INT32_MIN;
#pragma unroll
            for (int w = 0; w < HC_W; w++) {
                const uint32_t *o = xchg + ((((q * 3 + pass) * HC_W) + w) * 32 + lane) * 4;
                a0 += o[0]; a1 += o[1]; a2 += o[2];
                m0v = max(m0v, (int)o[0]); m1v = max(m1v, (int)o[1]); m2v = max(m2v, (int)o[2]);
            }
            if (pass == 0) {
                mx = m0v; mb = m1v; xs = m2v;   // a real logit is never INT32_MIN (|logit| < 2^30)
                krow = (long long)mx * (long long)c8 + 0x80000000ll;
            } else if (pass == 1) {
                S = a0;
                fd = make_freq_div(R, S);
            } else if (h == 0 && row < M) {
                const uint32_t rem = total - a0;   // to the first argmax (softmax_cdf.rs:125-127)
                const bool am_below = mb == mx, am_sym = !am_below && xs == mx;
                const uint32_t lo = a1 + (am_below ? rem : 0u);
                const uint32_t hi = lo + a2 + (am_sym ? rem : 0u);
                lohi[row] = make_uint2(lo, hi);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * HC_BN));
}

}  // namespace

void head_cdf_init() {
    cudaFuncSetAttribute(k_head_cdf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)HC_SMEM);
}

bool launch_head_cdf(const TcMatrix &A, const TcMatrix &B, int M, int V, int K, const uint32_t *sym,
                     const uint16_t *lut4k, uint32_t c8, uint32_t total, uint2 *lohi, int *err, cudaStream_t st) {
    if (M <= 0) return true;
    if (V % HC_BN != 0 || K % TC_BK != 0 || B.box_rows != HC_BN || A.box_rows != TC_BM) return false;
    const int n_mb = (M + TC_BM - 1) / TC_BM;
    const int grid = n_mb < sm_count() ? n_mb : sm_count();
    k_head_cdf<<<grid, HC_THREADS, HC_SMEM, st>>>(*reinterpret_cast<const CUtensorMap *>(A.map),
                                                  *reinterpret_cast<const CUtensorMap *>(B.map), M, V, K, sym, lut4k,
                                                  c8, total, lohi, err);
    return true;
}

}  // namespace czg
