// gemm_tc.cu -- int8 x int8 -> int32 "TN" GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8), operands staged by TMA, accumulator in TMEM.
//
// Computes the int8 linear layers of rust/src/linear.rs:12-31
// (out[m, n] = sum_k x[m, k] * W[n, k]) with the epilogues of gemm_mma.cu:
// requantisation (rust/src/model.rs:280-300), requantisation + ReGLU on
// interleaved gate/up columns (rust/src/reglu.rs:20-46), or raw int32.
//
// Persistent, warp-specialised kernel: one CTA per SM walks the 128 x BN output
// tiles (BN = 128 or 256) in a strided order.
//   warp 0 / lane 0  TMA producer: per 128-byte K block one box of A (128 rows)
//                    and one of B (BN rows), 128B-swizzled, into a ring of
//                    STAGES shared-memory stages (mbarriers full / empty);
//   warp 1           allocates TMEM; lane 0 issues 4 x tcgen05.mma (K = 32 each)
//                    per stage into one of two TMEM accumulators (2 x BN
//                    columns), tcgen05.commit frees the stage and, after the
//                    tile's last K block, hands the accumulator to the epilogue;
//   warps 2..9       epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 rows),
//                    the two warps of a quadrant each half of every 128-byte
//                    output slice; each converts its 64 bytes per row, writes
//                    them 64B-swizzled into its own staging buffer and stores
//                    them with TMA (cp.async.bulk.tensor, global <- shared),
//                    then releases the accumulator, so the epilogue of tile i
//                    overlaps the MMAs of tile i+1.
// Every mbarrier wait is bounded by a clock budget; on expiry the kernel sets
// kErrTimeout in the error word, every role stops, and TMEM is freed.
// No TMA load here uses cluster multicast.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int TC_BM = 128;
constexpr int TC_BK = 128;   // bytes of K per stage = one 128-byte swizzle row
constexpr int TC_EPI_WARPS = 8;   // two per TMEM lane quadrant, each taking half of a slice's columns
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_STAGE_OUT = 32 * 64;   // one epilogue warp's staging box: 32 rows x 64 bytes
constexpr long long kWaitBudget = 4000000000ll;   // clock cycles (about 2 s)

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bounded wait for the phase with the given parity; false when the budget ran
// out or (abort != nullptr) another role of the CTA has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, const volatile int *abort) {
    const uint32_t a = smem_addr(bar);
    const long long t0 = clock64();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if ((abort != nullptr && *abort) || clock64() - t0 > kWaitBudget) return false;
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// K-major, 128-byte swizzle smem matrix descriptor: rows 128 B apart, 8-row
// groups 1024 B apart (SBO = 64 x 16 B), LBO = 1, version 1, layout 2 = SW128.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)64u << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// kind::i8 instruction descriptor: D s32, A/B signed 8-bit, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(map), "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes (lane = row).  The load and
// its wait are one asm statement so that no use of the registers can be
// scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// Requantisation clamp(round_half_even(acc * mult / 2^shift), +-127) of
// model.rs:280-300 in three forms (mode):
//  2: |mult| < 2^(shift-1): A = the largest accumulator whose result is <= 127;
//     clamp(acc, -A, A) * mult fits int32 and lands exactly on +-127 at the clamp
//     (steps of the result are below 1/2), so no output clamp is needed;
//  1: clamp(acc, -A, A) with A * |mult| >= 128 * 2^shift (beyond it the result
//     saturates either way) fits int32; the output is clamped;
//  0: the 64-bit form.
struct Requant {
    int mult, shift, clamp_a, bias, mode;   // bias = 2^(shift-1) - 1
};

template <int RQ>
__device__ __forceinline__ int rq(int acc, const Requant &q) {
    if (RQ == 2) {
        const int x = min(max(acc, -q.clamp_a), q.clamp_a) * q.mult;
        return (x + q.bias + ((x >> q.shift) & 1)) >> q.shift;   // round half to even
    }
    if (RQ == 1) {
        const int x = min(max(acc, -q.clamp_a), q.clamp_a) * q.mult;
        return clamp127((x + q.bias + ((x >> q.shift) & 1)) >> q.shift);
    }
    return requant(acc, q.mult, q.shift);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// A slice: 128 output bytes per row, made from kAccCols accumulator columns; each of the
// two epilogue warps of a quadrant converts half of it (64 bytes, kOutCols elements).
template <int EPI>
struct EpiShape {
    static constexpr int kAccCols = EPI == kEpiInt32 ? 32 : (EPI == kEpiReglu ? 256 : 128);
    static constexpr int kOutCols = EPI == kEpiInt32 ? 16 : 64;
};

template <int BN, int STAGES, int EPI, int RQ>
__global__ void __launch_bounds__(TC_THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
          const __grid_constant__ CUtensorMap map_o, int M, int N, int K, Requant rqp, int *__restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int A_BYTES = TC_BM * TC_BK;
    constexpr int B_BYTES = BN * TC_BK;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int TMEM_COLS = 2 * BN;   // two accumulators
    constexpr int NCH = BN / EpiShape<EPI>::kAccCols;   // staging rows per tile
    uint8_t *stage_out = smem + STAGES * STAGE_BYTES;   // TC_EPI_WARPS warps x 2 buffers x 2 KB
    uint64_t *full = reinterpret_cast<uint64_t *>(stage_out + 2 * TC_EPI_WARPS * TC_STAGE_OUT);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = K / TC_BK;
    const int NT = N / BN;
    const int n_tiles = ((M + TC_BM - 1) / TC_BM) * NT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], TC_EPI_WARPS);
        }
        mbar_init(drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(TMEM_COLS));
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
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / NT) * TC_BM, n0 = (tile % NT) * BN;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], STAGE_BYTES);
                    tma_load_2d(sa, &map_a, &full[s], kb * TC_BK, m0);
                    tma_load_2d(sa + A_BYTES, &map_b, &full[s], kb * TC_BK, n0);
                }
            }
            if (!ok) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
                // let the loads already issued land before the CTA's shared memory goes away
                for (int k = max(0, it - STAGES); k < it; k++) mbar_wait(&full[k % STAGES], (k / STAGES) & 1, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            const uint32_t idesc = idesc_i8(TC_BM, BN);
            int it = 0, tc = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, tc++) {
                const int b = tc & 1;
                if (tc >= 2 && !mbar_wait(&tempty[b], ((tc >> 1) - 1) & 1, &abort_flag)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dt = tmem + (uint32_t)(b * BN);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
                    const uint64_t ad = smem_desc_sw128(sa);
                    const uint64_t bd = smem_desc_sw128(sa + A_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; k++)   // advance 32 bytes (2 x 16 B) inside the swizzle row
                        mma_i8(dt, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&tfull[b]);
            }
            if (!ok) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
            }
            // every MMA issued by this thread has completed once drain fires
            mma_commit(drain);
            mbar_wait(drain, 0, nullptr);
        }
    } else {   // epilogue warps 2..9
        const int q = warp & 3;            // TMEM lane quadrant = rows 32q .. 32q+31 of the tile
        const int hf = (warp - 2) >> 2;    // which half of each slice's columns
        uint8_t *sbuf0 = stage_out + (warp - 2) * 2 * TC_STAGE_OUT;
        int tc = 0, nb = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, tc++) {
            const int b = tc & 1;
            // every lane observes the accumulator's completion itself
            const bool got = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (tc >> 1) & 1, &abort_flag));
            if (!got) {
                if (lane == 0) {
                    atomicOr(err, kErrTimeout);
                    abort_flag = 1;
                }
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int m0 = (tile / NT) * TC_BM, n0 = (tile % NT) * BN;
            const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN);
            if (m0 + 32 * q >= M) {
                // no row of this warp exists: nothing to convert or store.  The staging
                // buffers must stay untouched here, since the stores of the previous
                // tile may still be reading them (wait_group.read counts only issued stores).
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
                continue;
            }
#pragma unroll 1
            for (int ch = 0; ch < NCH; ch++) {
                // staging buffer nb was handed to a TMA store two slices ago
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
                uint8_t *sb = sbuf0 + nb * TC_STAGE_OUT + lane * 64;   // this row's 64 output bytes
                constexpr int HC = EpiShape<EPI>::kAccCols / 2;          // accumulator columns of this warp
                const uint32_t tcol = tbase + (uint32_t)(ch * EpiShape<EPI>::kAccCols + hf * HC);
                // 64B swizzle of a 64-byte row: 16-byte chunk c lands at c ^ ((row >> 1) & 3)
                const int sw = (lane >> 1) & 3;
                if (EPI == kEpiInt32) {
                    uint32_t v[16];
                    tmem_ld16(tcol, v);
                    if (ch == NCH - 1) {   // the accumulator is free for the tile after next
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[b]);
                    }
#pragma unroll
                    for (int c = 0; c < 4; c++)
                        *reinterpret_cast<uint4 *>(sb + ((c ^ sw) << 4)) =
                            make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                } else {
                    // 32 accumulator columns at a time, converted straight into the staging row
                    constexpr int NG = HC / 32;
#pragma unroll 1
                    for (int gi = 0; gi < NG; gi++) {
                        uint32_t v[32];
                        tmem_ld32(tcol + 32 * gi, v);
                        if (ch == NCH - 1 && gi == NG - 1) {   // the accumulator is free for the tile after next
                            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&tempty[b]);
                        }
                        if (EPI == kEpiRequant) {   // 32 bytes: chunks 2gi, 2gi+1
                            uint32_t w[8];
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                w[j] = pack4(rq<RQ>((int)v[4 * j], rqp), rq<RQ>((int)v[4 * j + 1], rqp),
                                             rq<RQ>((int)v[4 * j + 2], rqp), rq<RQ>((int)v[4 * j + 3], rqp));
#pragma unroll
                            for (int hh = 0; hh < 2; hh++)
                                *reinterpret_cast<uint4 *>(sb + (((2 * gi + hh) ^ sw) << 4)) =
                                    make_uint4(w[4 * hh], w[4 * hh + 1], w[4 * hh + 2], w[4 * hh + 3]);
                        } else {   // ReGLU on (gate_j, up_j) = columns (2j, 2j+1) (reglu.rs:20-46): 16 bytes, chunk gi
                            int y[16];
#pragma unroll
                            for (int j = 0; j < 16; j++) {
                                const int gte = max(rq<RQ>((int)v[2 * j], rqp), 0);
                                const int x = gte * rq<RQ>((int)v[2 * j + 1], rqp);   // |x| <= 127 * 127
                                y[j] = (x + 63 + ((x >> 7) & 1)) >> 7;                  // |y| <= 126: no clamp
                            }
                            *reinterpret_cast<uint4 *>(sb + ((gi ^ sw) << 4)) =
                                make_uint4(pack4(y[0], y[1], y[2], y[3]), pack4(y[4], y[5], y[6], y[7]),
                                           pack4(y[8], y[9], y[10], y[11]), pack4(y[12], y[13], y[14], y[15]));
                        }
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {   // rows at or beyond M are clipped by the map
                    const int x = (EPI == kEpiReglu ? n0 / 2 : n0) + (2 * ch + hf) * EpiShape<EPI>::kOutCols;
                    tma_store_2d(&map_o, sbuf0 + nb * TC_STAGE_OUT, x, m0 + 32 * q);
                }
                nb ^= 1;
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

template <int BN>
struct TcCfg {
    static constexpr int kStages = BN == 256 ? 3 : 4;
    static constexpr size_t kSmem = 1024 + (size_t)kStages * (TC_BM + BN) * TC_BK + 2 * TC_EPI_WARPS * TC_STAGE_OUT +
                                    (2 * kStages + 5) * 8 + 16;
};

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

// TMA map of the output: [rows][cols] elements of elem_bytes, row pitch ld_bytes,
// stored in boxes of 64 bytes x 32 rows with the 64-byte swizzle.
bool make_out_map(CUtensorMap *map, void *base, uint64_t rows, uint64_t cols, uint64_t ld_bytes, int elem_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(64 / elem_bytes), 32};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims,
              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

Requant make_requant(int mult, int shift) {
    Requant q{mult, shift, 0, 0, 0};
    if (shift >= 1 && shift <= 24 && mult != 0) {
        const long long am = mult < 0 ? -(long long)mult : (long long)mult;
        q.bias = (1 << (shift - 1)) - 1;
        const long long a2 = ((255ll << (shift - 1)) + am - 1) / am - 1;   // largest a with a*|mult| < 127.5 * 2^shift
        const long long a1 = ((128ll << shift) / am) + 1;                 // |a * mult| >= 128 * 2^shift
        if (am < (1ll << (shift - 1)) && a2 * am + (1ll << (shift - 1)) < (1ll << 31)) {
            q.clamp_a = (int)a2;
            q.mode = 2;
        } else if (a1 * am + (1ll << (shift - 1)) < (1ll << 31)) {
            q.clamp_a = (int)a1;
            q.mode = 1;
        }
    }
    return q;
}

template <int BN, int EPI>
bool launch_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int mult, int shift, void *out,
               int ldo, int *err, cudaStream_t st) {
    alignas(64) CUtensorMap omap;
    const int eb = EPI == kEpiInt32 ? 4 : 1;
    const uint64_t cols = EPI == kEpiReglu ? (uint64_t)N / 2 : (uint64_t)N;
    if (!make_out_map(&omap, out, (uint64_t)M, cols, (uint64_t)ldo * eb, eb)) return false;
    const int tiles = ((M + TC_BM - 1) / TC_BM) * (N / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    const Requant q = make_requant(mult, shift);
    const CUtensorMap &ma = *reinterpret_cast<const CUtensorMap *>(A.map);
    const CUtensorMap &mb = *reinterpret_cast<const CUtensorMap *>(B.map);
    constexpr int S = TcCfg<BN>::kStages;
    if (EPI == kEpiInt32 || q.mode == 2)
        k_gemm_tc<BN, S, EPI, 2><<<grid, TC_THREADS, TcCfg<BN>::kSmem, st>>>(ma, mb, omap, M, N, K, q, err);
    else if (q.mode == 1)
        k_gemm_tc<BN, S, EPI, 1><<<grid, TC_THREADS, TcCfg<BN>::kSmem, st>>>(ma, mb, omap, M, N, K, q, err);
    else
        k_gemm_tc<BN, S, EPI, 0><<<grid, TC_THREADS, TcCfg<BN>::kSmem, st>>>(ma, mb, omap, M, N, K, q, err);
    return true;
}

template <int BN, int EPI>
void set_attr_epi() {
    cudaFuncSetAttribute(k_gemm_tc<BN, TcCfg<BN>::kStages, EPI, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TcCfg<BN>::kSmem);
    cudaFuncSetAttribute(k_gemm_tc<BN, TcCfg<BN>::kStages, EPI, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TcCfg<BN>::kSmem);
    cudaFuncSetAttribute(k_gemm_tc<BN, TcCfg<BN>::kStages, EPI, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TcCfg<BN>::kSmem);
}

template <int BN>
void set_attr() {
    set_attr_epi<BN, kEpiRequant>();
    set_attr_epi<BN, kEpiReglu>();
    set_attr_epi<BN, kEpiInt32>();
}

}  // namespace

int tc_bn_for(int N) {
    if (N % 256 == 0) return 256;
    if (N % 128 == 0) return 128;
    return 0;
}

bool tc_make_matrix(TcMatrix &m, const int8_t *base, uint64_t rows, uint64_t K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || K % TC_BK != 0 || rows == 0) return false;
    static_assert(sizeof(CUtensorMap) <= sizeof(m.map), "TcMatrix map storage too small");
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {K};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(reinterpret_cast<CUtensorMap *>(m.map), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                    const_cast<int8_t *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    m.rows = rows;
    m.K = K;
    m.box_rows = box_rows;
    return r == CUDA_SUCCESS;
}

void gemm_tc_init() {
    set_attr<128>();
    set_attr<256>();
}

bool launch_gemm_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int epi, int mult, int shift,
                    void *out, int ldo, int *err, cudaStream_t st) {
    if (M <= 0) return true;
    const int bn = tc_bn_for(N);
    if (bn == 0 || (epi == kEpiReglu && bn != 256)) return false;
    if (bn == 256) {
        if (epi == kEpiRequant) return launch_tc<256, kEpiRequant>(A, B, M, N, K, mult, shift, out, ldo, err, st);
        if (epi == kEpiReglu) return launch_tc<256, kEpiReglu>(A, B, M, N, K, mult, shift, out, ldo, err, st);
        return launch_tc<256, kEpiInt32>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    }
    if (epi == kEpiRequant) return launch_tc<128, kEpiRequant>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    return launch_tc<128, kEpiInt32>(A, B, M, N, K, mult, shift, out, ldo, err, st);
}

}  // namespace czg
