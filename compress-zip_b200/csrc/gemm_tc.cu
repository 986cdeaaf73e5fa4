// gemm_tc.cu -- int8 x int8 -> int32 "TN" GEMM on the 5th-generation tensor
// cores (tcgen05.mma kind::i8), operands staged by TMA, accumulator in TMEM.
//
// Computes the int8 linear layers of rust/src/linear.rs:12-31
// (out[m, n] = sum_k x[m, k] * W[n, k]) with the epilogues of gemm_mma.cu:
// requantisation (rust/src/model.rs:280-300), requantisation + ReGLU on
// interleaved gate/up columns (rust/src/reglu.rs:20-46), or raw int32.
//
// One CTA computes a 128 x BN output tile (BN = 128, 192 or 256):
//   warp 0 / lane 0  TMA producer: for each 128-byte K block, one box of A
//                    (128 rows) and one of B (BN rows), 128B-swizzled, into a
//                    ring of STAGES shared-memory stages (mbarrier full/empty);
//   warp 1 / lane 0  MMA issuer: 4 x tcgen05.mma (K = 32 each) per stage into
//                    one TMEM accumulator of BN columns; tcgen05.commit frees the
//                    stage and finally signals the epilogue;
//   warps 0..3       epilogue: warp w reads TMEM lanes 32w..32w+31 (its rows)
//                    with tcgen05.ld 32x32b and stores the converted row slice.
// Every mbarrier wait is bounded by a clock budget; on expiry the kernel sets
// kErrTimeout in the error word, skips the remaining work and frees its TMEM.
// No TMA load here uses cluster multicast.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int TC_BM = 128;
constexpr int TC_BK = 128;   // bytes of K per stage = one 128-byte swizzle row
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

// Bounded wait for the phase with the given parity; false when the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
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
        if (clock64() - t0 > kWaitBudget) return false;
    }
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

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(128, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M,
          int K, int mult, int shift, void *__restrict__ out, int ldo, int *__restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int A_BYTES = TC_BM * TC_BK;
    constexpr int B_BYTES = BN * TC_BK;
    constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int TMEM_COLS = BN <= 128 ? 128 : 256;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *done = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * BN;
    const int KB = K / TC_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // the whole warp allocates the accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // producer
        for (int kb = 0; kb < KB; kb++) {
            const int s = kb % STAGES;
            if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1)) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
                break;
            }
            uint8_t *sa = smem + s * STAGE_BYTES;
            mbar_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(sa, &map_a, &full[s], kb * TC_BK, m0);
            tma_load_2d(sa + A_BYTES, &map_b, &full[s], kb * TC_BK, n0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        const uint32_t idesc = idesc_i8(TC_BM, BN);
        bool ok = true;
        for (int kb = 0; kb < KB; kb++) {
            const int s = kb % STAGES;
            if (!mbar_wait(&full[s], (kb / STAGES) & 1)) {
                atomicOr(err, kErrTimeout);
                abort_flag = 1;
                ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
            const uint64_t ad = smem_desc_sw128(sa);
            const uint64_t bd = smem_desc_sw128(sa + A_BYTES);
#pragma unroll
            for (int k = 0; k < TC_BK / 32; k++)   // advance 32 bytes (2 x 16 B) inside the swizzle row
                mma_i8(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
            mma_commit(&empty[s]);
        }
        if (ok) mma_commit(done);
        else asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(done)) : "memory");
    }
    __syncwarp();

    // epilogue: all four warps
    const bool got = mbar_wait(done, 0);
    if (!got) atomicOr(err, kErrTimeout);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int row = m0 + warp * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    if (got && !abort_flag) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
            uint32_t v[16];
            tmem_ld16(trow + c, v);
            if (row < M) {
                if (EPI == kEpiInt32) {
                    int4 *o = reinterpret_cast<int4 *>(reinterpret_cast<int *>(out) + (size_t)row * ldo + n0 + c);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        o[q] = make_int4((int)v[4 * q], (int)v[4 * q + 1], (int)v[4 * q + 2], (int)v[4 * q + 3]);
                } else if (EPI == kEpiRequant) {
                    uint32_t w[4];
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        w[q] = 0;
#pragma unroll
                        for (int b = 0; b < 4; b++)
                            w[q] |= (uint32_t)(uint8_t)requant((int)v[4 * q + b], mult, shift) << (8 * b);
                    }
                    *reinterpret_cast<uint4 *>(reinterpret_cast<int8_t *>(out) + (size_t)row * ldo + n0 + c) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                } else {   // ReGLU on (gate_j, up_j) = columns (2j, 2j+1)
                    uint32_t w[2] = {0, 0};
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        int gte = max(requant((int)v[2 * j], mult, shift), 0);
                        int upv = requant((int)v[2 * j + 1], mult, shift);
                        w[j >> 2] |= (uint32_t)(uint8_t)clamp127(sra_rne32(gte * upv, 7)) << (8 * (j & 3));
                    }
                    *reinterpret_cast<uint2 *>(reinterpret_cast<int8_t *>(out) + (size_t)row * ldo + ((n0 + c) >> 1)) =
                        make_uint2(w[0], w[1]);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
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

template <int BN, int STAGES>
constexpr size_t tc_smem() {
    return 1024 + (size_t)STAGES * (TC_BM + BN) * TC_BK + (2 * STAGES + 1) * 8 + 16;
}

template <int BN, int STAGES, int EPI>
void launch_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int mult, int shift, void *out,
               int ldo, int *err, cudaStream_t st) {
    dim3 grid(N / BN, (M + TC_BM - 1) / TC_BM);
    k_gemm_tc<BN, STAGES, EPI><<<grid, 128, tc_smem<BN, STAGES>(), st>>>(
        *reinterpret_cast<const CUtensorMap *>(A.map), *reinterpret_cast<const CUtensorMap *>(B.map), M, K,
        mult, shift, out, ldo, err);
}

template <int BN, int STAGES>
void set_attr() {
    cudaFuncSetAttribute(k_gemm_tc<BN, STAGES, kEpiRequant>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem<BN, STAGES>());
    cudaFuncSetAttribute(k_gemm_tc<BN, STAGES, kEpiReglu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem<BN, STAGES>());
    cudaFuncSetAttribute(k_gemm_tc<BN, STAGES, kEpiInt32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem<BN, STAGES>());
}

template <int BN, int STAGES>
void dispatch_epi(int epi, const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int mult, int shift,
                  void *out, int ldo, int *err, cudaStream_t st) {
    if (epi == kEpiRequant) launch_tc<BN, STAGES, kEpiRequant>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    else if (epi == kEpiReglu) launch_tc<BN, STAGES, kEpiReglu>(A, B, M, N, K, mult, shift, out, ldo, err, st);
    else launch_tc<BN, STAGES, kEpiInt32>(A, B, M, N, K, mult, shift, out, ldo, err, st);
}

}  // namespace

int tc_bn_for(int N) {
    if (N % 256 == 0) return 256;
    if (N % 192 == 0) return 192;
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
    set_attr<128, 3>();
    set_attr<192, 2>();
    set_attr<256, 2>();
}

void launch_gemm_tc(const TcMatrix &A, const TcMatrix &B, int M, int N, int K, int epi, int mult, int shift,
                    void *out, int ldo, int *err, cudaStream_t st) {
    if (M <= 0) return;
    switch (tc_bn_for(N)) {
        case 256: dispatch_epi<256, 2>(epi, A, B, M, N, K, mult, shift, out, ldo, err, st); break;
        case 192: dispatch_epi<192, 2>(epi, A, B, M, N, K, mult, shift, out, ldo, err, st); break;
        default: dispatch_epi<128, 3>(epi, A, B, M, N, K, mult, shift, out, ldo, err, st); break;
    }
}

}  // namespace czg
