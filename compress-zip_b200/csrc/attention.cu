// attention.cu -- exact causal integer attention for whole chunks.
//
// Reference: gqa_attention_mqa_i8, rust/src/attention.rs:162-289, called for
// positions 0..n-1 of a chunk (rust/src/main.rs:212-217).  For query position p
// and head h the reference walks keys t = 0..p *in order* with an online softmax:
// when a score beats the running max m, the running sums are rescaled by
// exp(m - score) with rounding, so the result depends on where the prefix-max
// "records" fall.  Between records the weights w_t = exp(score_t - m) and the
// sums s += w, vacc += w * v are plain integer additions (u64 and wrapping i32),
// hence associative.  This kernel therefore:
//   * scores 32 keys at a time, one key per lane;
//   * finds the prefix max of the block with a warp scan (records = lanes whose
//     score beats the max of everything before them);
//   * adds record-free blocks in any order, and replays blocks that contain a
//     record key by key, applying each rescale where the reference does.
// Output: clamp(round_half_even(vacc / s)) per dimension (attention.rs:279-284).
//
// One CTA per chunk.  The chunk's rotated keys and values (kv rows, 128 B per
// position) are staged in shared memory when they fit.  Warps take (position,
// head) tasks longest-first from a shared counter.  Lane l owns output
// dimensions 2l and 2l+1.
#include "common.cuh"
#include "kernels.h"

namespace czg {
namespace {

constexpr int ATT_THREADS = 512;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int SMEM_KV_MAX = 1024;   // positions staged in shared memory

__device__ __forceinline__ int score_of(const uint32_t (&q)[16], const int8_t *krow, int mult) {
    const uint4 *k4 = reinterpret_cast<const uint4 *>(krow);
    int dot = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint4 kw = k4[i];
        dot = __dp4a((int)q[4 * i + 0], (int)kw.x, dot);
        dot = __dp4a((int)q[4 * i + 1], (int)kw.y, dot);
        dot = __dp4a((int)q[4 * i + 2], (int)kw.z, dot);
        dot = __dp4a((int)q[4 * i + 3], (int)kw.w, dot);
    }
    // attention.rs:236-245: round(dot >> 2), times score_mult (i64), round(>> 15)
    return sra_rne64_to32((long long)sra_rne32(dot, 2) * (long long)mult, 15);
}

// One warp: the query of head (qr = its 64 raw bytes) at position p against
// the keys 0..p of kv (rows of [k_rot 64 | v 64]); writes the 64 output bytes.
__device__ __forceinline__ void attend_query(const int8_t *__restrict__ qr, int p, int mult,
                                             const int8_t *__restrict__ sink_key,
                                             const int16_t *__restrict__ rope_cos,
                                             const int16_t *__restrict__ rope_sin,
                                             const uint16_t *lut, int8_t *qb, const int8_t *kv,
                                             int8_t *__restrict__ o) {
    const int lane = threadIdx.x & 31;
    const uint32_t coef = 378194u;   // ATTN_COEF_Q24, attention.rs:14-19
    // Q with RoPE and the NET_SHIFT rounding (attention.rs:53-83)
    {
        int x = qr[lane], y = qr[lane + 32];
        int cs = rope_cos[p * kHalfDim + lane], sn = rope_sin[p * kHalfDim + lane];
        qb[lane] = (int8_t)rope_q_round(x * cs - y * sn);
        qb[lane + 32] = (int8_t)rope_q_round(x * sn + y * cs);
    }
    __syncwarp();
    uint32_t q[16];
    {
        const uint4 *q4 = reinterpret_cast<const uint4 *>(qb);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint4 w = q4[i];
            q[4 * i] = w.x; q[4 * i + 1] = w.y; q[4 * i + 2] = w.z; q[4 * i + 3] = w.w;
        }
    }
    __syncwarp();

    int m = INT32_MIN;
    unsigned long long s = 0;
    uint32_t va0 = 0, va1 = 0;   // wrapping i32 accumulators of dims 2*lane, 2*lane+1
    if (sink_key != nullptr) {   // attention.rs:211-224: sink score is the first max
        m = score_of(q, sink_key, mult);
        s = 65535ull;
    }

    for (int kb = 0; kb <= p; kb += 32) {
        const int t = kb + lane;
        const bool valid = t <= p;
        const int sc = valid ? score_of(q, kv + (size_t)t * 128, mult) : INT32_MIN;
        int incl = sc;   // inclusive prefix max over the block, in key order
#pragma unroll
        for (int o2 = 1; o2 < 32; o2 <<= 1) {
            int u = __shfl_up_sync(0xffffffffu, incl, o2);
            if (lane >= o2) incl = max(incl, u);
        }
        incl = max(incl, m);
        int prev = __shfl_up_sync(0xffffffffu, incl, 1);
        if (lane == 0) prev = m;
        const bool rec = valid && sc > prev;
        // weight against the max in force after this key (attention.rs:266-268)
        const uint32_t w = valid ? exp_q16((int)((uint32_t)sc - (uint32_t)incl), lut, coef) : 0u;
        // rescale factor applied at this key when it sets a new max (attention.rs:248-263)
        const uint32_t e = (rec && prev != INT32_MIN)
                               ? exp_q16((int)((uint32_t)prev - (uint32_t)sc), lut, coef) : 0u;
        const uint32_t recs = __ballot_sync(0xffffffffu, rec);
        const int nvalid = min(32, p - kb + 1);
        const int8_t *vbase = kv + (size_t)kb * 128 + 64 + 2 * lane;
        if (recs == 0) {
            uint32_t ws = w;
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o2);
            s += ws;
            for (int j = 0; j < nvalid; j++) {
                uint32_t wj = __shfl_sync(0xffffffffu, w, j);
                uint32_t vv = *reinterpret_cast<const uint16_t *>(vbase + (size_t)j * 128);
                va0 += wj * (uint32_t)sext8(vv, 0);
                va1 += wj * (uint32_t)sext8(vv, 1);
            }
        } else {
            for (int j = 0; j < nvalid; j++) {
                uint32_t wj = __shfl_sync(0xffffffffu, w, j);
                uint32_t ej = __shfl_sync(0xffffffffu, e, j);
                if (((recs >> j) & 1u) && ej != 0u) {
                    s = (s * ej + 0x8000ull) >> 16;
                    long long p0 = (long long)(int)va0 * (long long)ej;
                    long long p1 = (long long)(int)va1 * (long long)ej;
                    p0 += p0 >= 0 ? (1ll << 15) : -(1ll << 15);
                    p1 += p1 >= 0 ? (1ll << 15) : -(1ll << 15);
                    va0 = (uint32_t)(int)(p0 >> 16);
                    va1 = (uint32_t)(int)(p1 >> 16);
                }
                s += wj;
                uint32_t vv = *reinterpret_cast<const uint16_t *>(vbase + (size_t)j * 128);
                va0 += wj * (uint32_t)sext8(vv, 0);
                va1 += wj * (uint32_t)sext8(vv, 1);
            }
        }
        m = __shfl_sync(0xffffffffu, incl, 31);
    }
    const unsigned long long den = s == 0 ? 1ull : s;
    uint16_t pk = (uint16_t)(uint8_t)clamp127(div_rne_s32_u64((int)va0, den)) |
                  ((uint16_t)(uint8_t)clamp127(div_rne_s32_u64((int)va1, den)) << 8);
    *reinterpret_cast<uint16_t *>(o + 2 * lane) = pk;
}

template <bool KV_SMEM>
__global__ void __launch_bounds__(ATT_THREADS, 1)
k_attention(const int8_t *__restrict__ qkv, int ldq, const int8_t *__restrict__ kv_g,
            const int *__restrict__ chunk_row0, const int *__restrict__ chunk_len, int n_heads,
            const int32_t *__restrict__ score_mult, const int8_t *__restrict__ sink_key,
            const int16_t *__restrict__ rope_cos, const int16_t *__restrict__ rope_sin,
            const uint16_t *__restrict__ lut_g, int8_t *__restrict__ out, int ldo) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint16_t lut[256];
    __shared__ int task_ctr;
    __shared__ __align__(16) int8_t qbuf[ATT_WARPS][64];

    const int c = blockIdx.x;
    const int r0 = chunk_row0[c], n = chunk_len[c];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < 256; i += ATT_THREADS) lut[i] = lut_g[i];
    if (tid == 0) task_ctr = 0;

    const int8_t *kv;
    if (KV_SMEM) {
        uint4 *dst = reinterpret_cast<uint4 *>(smem);
        const uint4 *src = reinterpret_cast<const uint4 *>(kv_g + (size_t)r0 * 128);
        for (int i = tid; i < n * 8; i += ATT_THREADS) dst[i] = src[i];
        kv = reinterpret_cast<const int8_t *>(smem);
    } else {
        kv = kv_g + (size_t)r0 * 128;
    }
    __syncthreads();

    const int n_tasks = n * n_heads;
    for (;;) {
        int task = 0;
        if (lane == 0) task = atomicAdd(&task_ctr, 1);
        task = __shfl_sync(0xffffffffu, task, 0);
        if (task >= n_tasks) break;
        const int p = n - 1 - task / n_heads;   // longest first
        const int h = task % n_heads;
        attend_query(qkv + (size_t)(r0 + p) * ldq + h * 64, p, score_mult[h], sink_key, rope_cos, rope_sin,
                     lut, qbuf[warp], kv, out + (size_t)(r0 + p) * ldo + h * 64);
    }
}

// Decode step: row r of the batch is a stream at position p; its keys are the
// rows 0..p of its KV cache (kvc + r * cache_ld).  One warp per (row, head).
__global__ void __launch_bounds__(256)
k_attention_decode(const int8_t *__restrict__ qkv, int ldq, const int8_t *__restrict__ kvc,
                   size_t cache_ld, int M, int p, int n_heads, const int32_t *__restrict__ score_mult,
                   const int8_t *__restrict__ sink_key, const int16_t *__restrict__ rope_cos,
                   const int16_t *__restrict__ rope_sin, const uint16_t *__restrict__ lut_g,
                   int8_t *__restrict__ out, int ldo) {
    __shared__ uint16_t lut[256];
    __shared__ __align__(16) int8_t qbuf[8][64];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = lut_g[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const int task = blockIdx.x * 8 + warp;
    if (task >= M * n_heads) return;
    const int r = task / n_heads, h = task % n_heads;
    attend_query(qkv + (size_t)r * ldq + h * 64, p, score_mult[h], sink_key, rope_cos, rope_sin, lut,
                 qbuf[warp], kvc + (size_t)r * cache_ld, out + (size_t)r * ldo + h * 64);
}

}  // namespace

void launch_attention_decode(const int8_t *qkv, int ldq, const int8_t *kvc, size_t cache_ld, int M, int p,
                             int n_heads, const int32_t *score_mult, const int8_t *sink_key,
                             const int16_t *rope_cos, const int16_t *rope_sin, const uint16_t *lut,
                             int8_t *out, int ldo, cudaStream_t st) {
    if (M == 0) return;
    const int tasks = M * n_heads;
    k_attention_decode<<<(tasks + 7) / 8, 256, 0, st>>>(qkv, ldq, kvc, cache_ld, M, p, n_heads, score_mult,
                                                        sink_key, rope_cos, rope_sin, lut, out, ldo);
}

void attention_init() {
    cudaFuncSetAttribute(k_attention<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         SMEM_KV_MAX * 128);
}

void launch_attention(const int8_t *qkv, int ldq, const int8_t *kv, const int *chunk_row0,
                      const int *chunk_len, int n_chunks, int max_len, int n_heads,
                      const int32_t *score_mult, const int8_t *sink_key, const int16_t *rope_cos,
                      const int16_t *rope_sin, const uint16_t *lut, int8_t *out, int ldo,
                      cudaStream_t st) {
    if (n_chunks == 0) return;
    if (max_len <= SMEM_KV_MAX) {
        size_t smem = (size_t)max_len * 128;
        k_attention<true><<<n_chunks, ATT_THREADS, smem, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut, out, ldo);
    } else {
        k_attention<false><<<n_chunks, ATT_THREADS, 0, st>>>(
            qkv, ldq, kv, chunk_row0, chunk_len, n_heads, score_mult, sink_key, rope_cos, rope_sin,
            lut, out, ldo);
    }
}

}  // namespace czg
