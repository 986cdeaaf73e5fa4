// gemm_tc.cu -- int8 x int8 -> int32 "TN" GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8), operands staged by TMA, accumulator in TMEM.
//
// Computes the int8 linear layers of rust/src/linear.rs:12-31
// (out[m, n] = sum_k x[m, k] * W[n, k]) with one of four epilogues:
// requantisation (rust/src/model.rs:280-300), requantisation + ReGLU on
// interleaved gate/up columns (rust/src/reglu.rs:20-46), raw int32, or the QKV
// projection's requantisation with the key rotated (rust/src/attention.rs:29-50)
// and the key and value written straight into the attention's per-chunk layout.
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
#include <cmath>
#include <cstdlib>

#include "kernels.h"
#include "tc_common.cuh"

namespace czg {
namespace {

constexpr int TC_EPI_WARPS = 8;   // two per TMEM lane quadrant, each taking half of a slice's columns
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_STAGE_OUT = 32 * 64;   // one epilogue warp's staging box: 32 rows x 64 bytes

// Requantisation clamp(round_half_even(acc * mult / 2^shift), +-127) of
// model.rs:280-300 in four forms (mode):
//  3: mode 2's clamp, then the product and its rounding in one FP32 fused
//     multiply-add on the biased accumulator (common.cuh, kM1Bits): the result is
//     the float M1 + requant, whose low byte is the int8 output (chosen when the
//     clamp bound is below 2^22 and mult / 2^shift, M1 - M1 * mult / 2^shift are
//     exact floats);
//  2: |mult| < 2^(shift-1): A = the largest accumulator whose result is <= 127;
//     clamp(acc, -A, A) * mult fits int32 and lands exactly on +-127 at the clamp
//     (steps of the result are below 1/2), so no output clamp is needed;
//  1: clamp(acc, -A, A) with A * |mult| >= 128 * 2^shift (beyond it the result
//     saturates either way) fits int32; the output is clamped;
//  0: the 64-bit form.
struct Requant {
    int mult, shift, clamp_a, bias, mode;   // bias = 2^(shift-1) - 1
    float mf, c2;                           // mode 3: mult / 2^shift, M1 - M1 * mult / 2^shift
};

// mode 3: bits of the float M1 + requant(acc)
// (the clamp to +-A and the bias as max(acc + bits(M1), bits(M1) - A), one fused
// add-max, then min(., bits(M1) + A); |acc| < 2^29 keeps the sum inside int32)
__device__ __forceinline__ uint32_t rq_flt(int acc, const Requant &q) {
    const int b = min(__viaddmax_s32(acc, (int)kM1Bits, (int)kM1Bits - q.clamp_a), (int)kM1Bits + q.clamp_a);
    return __float_as_uint(__fmaf_rn(__int_as_float(b), q.mf, q.c2));
}
// mode 3 with mult > 0, a ReGLU gate: the float M1 + max(requant(acc), 0), which is
// M1 + requant(max(acc, 0)) since requant is then non-decreasing with requant(0) = 0
__device__ __forceinline__ float rq_gate_pos(int acc, const Requant &q) {
    const int b = min(__viaddmax_s32(acc, (int)kM1Bits, (int)kM1Bits), (int)kM1Bits + q.clamp_a);
    return __fmaf_rn(__int_as_float(b), q.mf, q.c2);
}

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

// kEpiRequantKv, key slice: the row's 64 key bytes (staged, 64B-swizzled) rotated
// (attention.rs:29-50, as k_kv_prep_split) and stored as the split layout's K row
// (word W = dims 4W..4W+3 at word 4 (W % 4) + W / 4) with four 16-byte stores.
__device__ __forceinline__ void kv_store_key(const uint8_t *srow, int sw, const int16_t *__restrict__ rc,
                                             const int16_t *__restrict__ rs, int8_t *dst) {
    uint32_t kw[16];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 v = *reinterpret_cast<const uint4 *>(srow + ((c ^ sw) << 4));
        kw[4 * c] = v.x; kw[4 * c + 1] = v.y; kw[4 * c + 2] = v.z; kw[4 * c + 3] = v.w;
    }
    uint32_t cw[16], sn[16];   // the position's 32 cos and 32 sin values, two per word
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(rc) + c), b = __ldg(reinterpret_cast<const uint4 *>(rs) + c);
        cw[4 * c] = a.x; cw[4 * c + 1] = a.y; cw[4 * c + 2] = a.z; cw[4 * c + 3] = a.w;
        sn[4 * c] = b.x; sn[4 * c + 1] = b.y; sn[4 * c + 2] = b.z; sn[4 * c + 3] = b.w;
    }
    uint32_t ow[16];
#pragma unroll
    for (int W = 0; W < 8; W++) {   // dims 4W..4W+3 and their partners + 32
        uint32_t xw = 0, yw = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int i = 4 * W + b;
            const int x = sext8(kw[W], b), y = sext8(kw[W + 8], b);
            const int c = (int)(int16_t)(cw[i >> 1] >> (16 * (i & 1))), s = (int)(int16_t)(sn[i >> 1] >> (16 * (i & 1)));
            xw |= (uint32_t)(uint8_t)rope_k_round(x * c - y * s) << (8 * b);
            yw |= (uint32_t)(uint8_t)rope_k_round(x * s + y * c) << (8 * b);
        }
        ow[4 * (W & 3) + (W >> 2)] = xw;
        ow[4 * ((W + 8) & 3) + ((W + 8) >> 2)] = yw;
    }
    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int c = 0; c < 4; c++) d4[c] = make_uint4(ow[4 * c], ow[4 * c + 1], ow[4 * c + 2], ow[4 * c + 3]);
}

template <int BN, int STAGES, int EPI, int RQ>
__global__ void __launch_bounds__(TC_THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
          const __grid_constant__ CUtensorMap map_o, int M, int N, int K, Requant rqp, int *__restrict__ err,
          KvSplit kvs) {
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
    // the setup above overlaps the previous kernel under a PDL launch; the operands
    // and the output buffer are touched only from here on
    pdl_wait();
    pdl_trigger();

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
                        if (EPI == kEpiRequant || EPI == kEpiRequantKv) {   // 32 bytes: chunks 2gi, 2gi+1
                            uint32_t w[8];
#pragma unroll
                            for (int j = 0; j < 8; j++) {
                                if (RQ == 3)
                                    w[j] = pack4(rq_flt((int)v[4 * j], rqp), rq_flt((int)v[4 * j + 1], rqp),
                                                 rq_flt((int)v[4 * j + 2], rqp), rq_flt((int)v[4 * j + 3], rqp));
                                else
                                    w[j] = pack4(rq<RQ>((int)v[4 * j], rqp), rq<RQ>((int)v[4 * j + 1], rqp),
                                                 rq<RQ>((int)v[4 * j + 2], rqp), rq<RQ>((int)v[4 * j + 3], rqp));
                            }
#pragma unroll
                            for (int hh = 0; hh < 2; hh++)
                                *reinterpret_cast<uint4 *>(sb + (((2 * gi + hh) ^ sw) << 4)) =
                                    make_uint4(w[4 * hh], w[4 * hh + 1], w[4 * hh + 2], w[4 * hh + 3]);
                        } else {   // ReGLU on (gate_j, up_j) = columns (2j, 2j+1) (reglu.rs:20-46): 16 bytes, chunk gi
                            int y[16];
                            if (RQ == 3 && rqp.mult > 0) {   // y = M1 + rne(g * u / 128), g = max(gate, 0), in FP32, exact
#pragma unroll
                                for (int j = 0; j < 16; j++) {
                                    const float gate = __fsub_rn(rq_gate_pos((int)v[2 * j], rqp), kM1);
                                    const float ub = __uint_as_float(rq_flt((int)v[2 * j + 1], rqp));
                                    const float u128 = __fmaf_rn(ub, 0.0078125f, -98304.0f);   // (ub - M1) / 128
                                    y[j] = __float_as_int(__fmaf_rn(gate, u128, kM1));
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < 16; j++) {
                                    if (RQ == 3) {
                                        const float gb = __uint_as_float(rq_flt((int)v[2 * j], rqp));
                                        const float ub = __uint_as_float(rq_flt((int)v[2 * j + 1], rqp));
                                        const float gate = fmaxf(__fsub_rn(gb, kM1), 0.0f);
                                        const float u128 = __fmaf_rn(ub, 0.0078125f, -98304.0f);
                                        y[j] = __float_as_int(__fmaf_rn(gate, u128, kM1));
                                    } else {
                                        const int gte = max(rq<RQ>((int)v[2 * j], rqp), 0);
                                        const int x = gte * rq<RQ>((int)v[2 * j + 1], rqp);   // |x| <= 127 * 127
                                        y[j] = (x + 63 + ((x >> 7) & 1)) >> 7;                  // |y| <= 126: no clamp
                                    }
                                }
                            }
                            *reinterpret_cast<uint4 *>(sb + ((gi ^ sw) << 4)) =
                                make_uint4(pack4(y[0], y[1], y[2], y[3]), pack4(y[4], y[5], y[6], y[7]),
                                           pack4(y[8], y[9], y[10], y[11]), pack4(y[12], y[13], y[14], y[15]));
                        }
                    }
                }
                if (EPI == kEpiRequantKv && n0 + ch * EpiShape<EPI>::kAccCols == kvs.d) {
                    // the key (hf 0) and value (hf 1) columns go to the split layout instead
                    // of the output; each warp reads only its own staging buffer, so the two
                    // need no barrier (splitting the key between them behind one was slower)
                    __syncwarp();
                    const int row = m0 + 32 * q + lane;
                    uint32_t voff = 0;   // byte offset in kv of this row's value bytes (dim 0)
                    if (row < M) {
                        const int c = kvs.rowchunk[row], r0 = kvs.chunk_row0[c];
                        const int p = row - r0;
                        const size_t base = ((size_t)r0 + 32 * (size_t)c) * 128;
                        if (hf == 0) {
                            kv_store_key(sbuf0 + nb * TC_STAGE_OUT + lane * 64, (lane >> 1) & 3,
                                         kvs.rope_cos + p * kHalfDim, kvs.rope_sin + p * kHalfDim,
                                         kvs.kv + base + (size_t)p * 64);
                        } else {
                            const int npad = (kvs.chunk_len[c] + 31) & ~31;
                            // the V tile of key p (a multiple of 128 bytes) with p % 32 in the low bits
                            voff = (uint32_t)(base + (size_t)npad * 64 + (size_t)(p >> 5) * 2048) | (uint32_t)(p & 31);
                        }
                    }
                    if (hf == 1) {   // value dims 2l, 2l + 1 of each row into its V tile (vt_byte, common.cuh)
                        const uint8_t *sv = sbuf0 + nb * TC_STAGE_OUT;
                        const int nrow = min(32, M - (m0 + 32 * q));
#pragma unroll 4
                        for (int r = 0; r < nrow; r++) {
                            const uint32_t o = __shfl_sync(0xffffffffu, voff, r);
                            const int kp = (int)(o & 31u);
                            int8_t *vt = kvs.kv + (o & ~31u);
                            const uint16_t v2 = *reinterpret_cast<const uint16_t *>(
                                sv + r * 64 + (((lane >> 3) ^ ((r >> 1) & 3)) << 4) + 2 * (lane & 7));
                            vt[vt_byte(kp, 2 * lane)] = (int8_t)(v2 & 0xFFu);
                            vt[vt_byte(kp, 2 * lane + 1)] = (int8_t)(v2 >> 8);
                        }
                    }
                    __syncwarp();   // the staging buffer stays this warp's: no store was issued
                    continue;
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

template <int BN>
struct TcCfg {
    static constexpr int kStages = BN == 256 ? 3 : 4;
    static constexpr size_t kSmem = 1024 + (size_t)kStages * (TC_BM + BN) * TC_BK + 2 * TC_EPI_WARPS * TC_STAGE_OUT +
                                    (2 * kStages + 5) * 8 + 16;
};

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
    Requant q{mult, shift, 0, 0, 0, 0.0f, 0.0f};
    if (shift >= 1 && shift <= 24 && mult != 0) {
        const long long am = mult < 0 ? -(long long)mult : (long long)mult;
        q.bias = (1 << (shift - 1)) - 1;
        const long long a2 = ((255ll << (shift - 1)) + am - 1) / am - 1;   // largest a with a*|mult| < 127.5 * 2^shift
        const long long a1 = ((128ll << shift) / am) + 1;                 // |a * mult| >= 128 * 2^shift
        if (am < (1ll << (shift - 1)) && a2 * am + (1ll << (shift - 1)) < (1ll << 31)) {
            q.clamp_a = (int)a2;
            q.mode = 2;
            const double mfd = std::ldexp((double)mult, -shift);
            const double c2d = 12582912.0 - 12582912.0 * mfd;
            if (a2 < (1ll << 22) && (double)(float)mfd == mfd && (double)(float)c2d == c2d &&
                std::getenv("CZG_INT_REQUANT") == nullptr) {
                q.mf = (float)mfd;
                q.c2 = (float)c2d;
                q.mode = 3;
            }
        } else if (a1 * am + (1ll << (shift - 1)) < (1ll << 31)) {
            q.clamp_a = (int)a1;
            q.mode = 1;
        }
    }
    return q;
}

template <int BN, int EPI>
bool launch_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int mult, int shift, void *out,
               int ldo, int *err, cudaStream_t st, const KvSplit &kvs = KvSplit{}) {
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
    // the FP32 form adds bits(M1) to the raw accumulator: |acc| <= K * 128 * 127 < 2^29
    const bool fp32 = q.mode == 3 && (long long)K * 16256 < (1ll << 29);
    if (EPI != kEpiInt32 && fp32)
        launch_k(k_gemm_tc<BN, S, EPI, 3>, grid, TC_THREADS, TcCfg<BN>::kSmem, st, ma, mb, omap, M, N, K, q, err, kvs);
    else if (EPI == kEpiInt32 || q.mode == 2 || q.mode == 3)
        launch_k(k_gemm_tc<BN, S, EPI, 2>, grid, TC_THREADS, TcCfg<BN>::kSmem, st, ma, mb, omap, M, N, K, q, err, kvs);
    else if (q.mode == 1)
        launch_k(k_gemm_tc<BN, S, EPI, 1>, grid, TC_THREADS, TcCfg<BN>::kSmem, st, ma, mb, omap, M, N, K, q, err, kvs);
    else
        launch_k(k_gemm_tc<BN, S, EPI, 0>, grid, TC_THREADS, TcCfg<BN>::kSmem, st, ma, mb, omap, M, N, K, q, err, kvs);
    return true;
}

template <int BN, int EPI>
void set_attr_epi() {
    cudaFuncSetAttribute(k_gemm_tc<BN, TcCfg<BN>::kStages, EPI, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)TcCfg<BN>::kSmem);
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
    set_attr_epi<BN, kEpiRequantKv>();
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

bool requant_fp32(int mult, int shift, float *mf, float *c2, int *clamp_a) {
    const Requant q = make_requant(mult, shift);
    if (q.mode != 3) return false;
    *mf = q.mf;
    *c2 = q.c2;
    *clamp_a = q.clamp_a;
    return true;
}

void gemm_tc_init() {
    set_attr<128>();
    set_attr<256>();
}

bool launch_gemm_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int epi, int mult, int shift,
                    void *out, int ldo, int *err, cudaStream_t st, const KvSplit *kvs) {
    if (M <= 0) return true;
    const int bn = tc_bn_for(N);
    if (bn == 0 || (epi == kEpiReglu && bn != 256)) return false;
    if (epi == kEpiRequantKv) {   // the key/value slice must be one whole 128-column slice
        if (kvs == nullptr || kvs->d % 128 != 0 || N != kvs->d + 128) return false;
        return bn == 256 ? launch_tc<256, kEpiRequantKv>(A, B, M, N, K, mult, shift, out, ldo, err, st, *kvs)
                         : launch_tc<128, kEpiRequantKv>(A, B, M, N, K, mult, shift, out, ldo, err, st, *kvs);
    }
    if (bn == 256) {
        if (epi == kEpiRequant) return launch_tc<256, kEpiRequant>(A, B, M, N, K, mult, shift, out, ldo, err, st);
        if (epi == kEpiReglu) return launch_tc<256, kEpiReglu>(A, B, M, N, K, mult, shift, out, ldo, err, st);
        return launch_tc<256, kEpiInt32>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    }
    if (epi == kEpiRequant) return launch_tc<128, kEpiRequant>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    return launch_tc<128, kEpiInt32>(A, B, M, N, K, mult, shift, out, ldo, err, st);
}

}  // namespace czg
