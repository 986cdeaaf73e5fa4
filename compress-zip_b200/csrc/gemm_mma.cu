// gemm_mma.cu -- int8 x int8 -> int32 "TN" GEMM with fused epilogues, built on
// warp-level mma.sync (m16n8k32 .s8) and a cp.async 3-stage pipeline.
//
// Computes the int8 linear layers of rust/src/linear.rs:12-31
// (out[m, n] = sum_k x[m, k] * W[n, k]) followed by the requantisation of
// rust/src/model.rs:280-300 and, for the FFN up projection, ReGLU
// (rust/src/reglu.rs:20-46).  Accumulation is exact: |acc| <= 127^2 * K < 2^31.
//
// Tile 128x128x64, 8 warps (2 along M x 4 along N), warp tile 64x32.
// Shared-memory rows are 64 bytes; 16-byte chunks are XOR-swizzled by
// ((row >> 1) & 3) so the fragment loads of a warp hit 32 distinct banks.
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3, THREADS = 256;
constexpr int TILE_BYTES = BM * BK;   // one operand tile per stage (BM == BN)

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ int swz(int row, int chunk) { return chunk ^ ((row >> 1) & 3); }

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Copy one 128x64 tile (rows r0.., k-block kb) of a row-major [rows][K] matrix.
__device__ __forceinline__ void load_tile(uint8_t *sm, const int8_t *g, int r0, int K, int kb, int tid) {
#pragma unroll
    for (int it = 0; it < 2; it++) {
        int idx = tid + it * THREADS;
        int row = idx >> 2, ch = idx & 3;
        const int8_t *src = g + (size_t)(r0 + row) * K + kb * BK + ch * 16;
        cp_async16(smem_u32(sm + row * BK + swz(row, ch) * 16), src);
    }
}

template <int EPI>
__global__ void __launch_bounds__(THREADS) k_gemm(const int8_t *__restrict__ A,
                                                  const int8_t *__restrict__ B, int M, int N, int K,
                                                  int mult, int shift, void *__restrict__ out,
                                                  int ldo) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * TILE_BYTES;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 2, wn = warp & 3;
    const int g = lane >> 2, tig = lane & 3;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int KB = K / BK;

    int acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int k = 0; k < 4; k++) acc[i][j][k] = 0;

#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < KB) {
            load_tile(sA + s * TILE_BYTES, A, m0, K, s, tid);
            load_tile(sB + s * TILE_BYTES, B, n0, K, s, tid);
        }
        cp_commit();
    }

    for (int kb = 0; kb < KB; kb++) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        int nk = kb + STAGES - 1;
        if (nk < KB) {
            int s = nk % STAGES;
            load_tile(sA + s * TILE_BYTES, A, m0, K, nk, tid);
            load_tile(sB + s * TILE_BYTES, B, n0, K, nk, tid);
        }
        cp_commit();

        const uint8_t *tA = sA + (kb % STAGES) * TILE_BYTES;
        const uint8_t *tB = sB + (kb % STAGES) * TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
            uint32_t af[4][4], bf[4][2];
#pragma unroll
            for (int mi = 0; mi < 4; mi++) {
                int r = wm * 64 + mi * 16 + g;
                af[mi][0] = *reinterpret_cast<const uint32_t *>(tA + r * BK + swz(r, 2 * kk) * 16 + tig * 4);
                af[mi][1] = *reinterpret_cast<const uint32_t *>(tA + (r + 8) * BK + swz(r + 8, 2 * kk) * 16 + tig * 4);
                af[mi][2] = *reinterpret_cast<const uint32_t *>(tA + r * BK + swz(r, 2 * kk + 1) * 16 + tig * 4);
                af[mi][3] = *reinterpret_cast<const uint32_t *>(tA + (r + 8) * BK + swz(r + 8, 2 * kk + 1) * 16 + tig * 4);
            }
#pragma unroll
            for (int ni = 0; ni < 4; ni++) {
                int n = wn * 32 + ni * 8 + g;
                bf[ni][0] = *reinterpret_cast<const uint32_t *>(tB + n * BK + swz(n, 2 * kk) * 16 + tig * 4);
                bf[ni][1] = *reinterpret_cast<const uint32_t *>(tB + n * BK + swz(n, 2 * kk + 1) * 16 + tig * 4);
            }
#pragma unroll
            for (int mi = 0; mi < 4; mi++)
#pragma unroll
                for (int ni = 0; ni < 4; ni++) mma_s8(acc[mi][ni], af[mi], bf[ni]);
        }
    }
    cp_wait<0>();

    // epilogue: thread holds (row g | g+8, cols 2*tig, 2*tig+1) of each 16x8 tile
#pragma unroll
    for (int mi = 0; mi < 4; mi++)
#pragma unroll
        for (int half = 0; half < 2; half++) {
            int row = m0 + wm * 64 + mi * 16 + g + half * 8;
            if (row >= M) continue;
#pragma unroll
            for (int ni = 0; ni < 4; ni++) {
                int col = n0 + wn * 32 + ni * 8 + tig * 2;
                int c0 = acc[mi][ni][2 * half], c1 = acc[mi][ni][2 * half + 1];
                if (EPI == kEpiInt32) {
                    int *o = reinterpret_cast<int *>(out) + (size_t)row * ldo + col;
                    *reinterpret_cast<int2 *>(o) = make_int2(c0, c1);
                } else if (EPI == kEpiRequant) {
                    int8_t *o = reinterpret_cast<int8_t *>(out) + (size_t)row * ldo + col;
                    uint16_t v = (uint16_t)(uint8_t)requant(c0, mult, shift) |
                                 ((uint16_t)(uint8_t)requant(c1, mult, shift) << 8);
                    *reinterpret_cast<uint16_t *>(o) = v;
                } else {   // ReGLU: even column = gate_j, odd column = up_j, j = col / 2
                    int gte = max(requant(c0, mult, shift), 0);
                    int upv = requant(c1, mult, shift);
                    int8_t *o = reinterpret_cast<int8_t *>(out) + (size_t)row * ldo + (col >> 1);
                    *o = (int8_t)clamp127(sra_rne32(gte * upv, 7));
                }
            }
        }
}

}  // namespace

void launch_gemm(const int8_t *A, const int8_t *B, int M, int N, int K, int epi, int mult,
                 int shift, void *out, int ldo, cudaStream_t st) {
    if (M <= 0) return;
    dim3 grid(N / BN, (M + BM - 1) / BM);
    size_t smem = 2 * STAGES * TILE_BYTES;
    switch (epi) {
        case kEpiRequant:
            k_gemm<kEpiRequant><<<grid, THREADS, smem, st>>>(A, B, M, N, K, mult, shift, out, ldo);
            break;
        case kEpiReglu:
            k_gemm<kEpiReglu><<<grid, THREADS, smem, st>>>(A, B, M, N, K, mult, shift, out, ldo);
            break;
        default:
            k_gemm<kEpiInt32><<<grid, THREADS, smem, st>>>(A, B, M, N, K, mult, shift, out, ldo);
            break;
    }
}

}  // namespace czg
