// common.cuh -- device integer arithmetic shared by the sm_100a kernels.
//
// Every helper reproduces the exact integer semantics of the reference crate
// (carsonpo/compress-zip, rust/src), cited per function; Rust release builds
// wrap on overflow, so accumulators that may wrap are kept in uint32_t.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include <utility>

#include "kernels.h"

namespace czg {

constexpr int kHeadDim = 64;
constexpr int kHalfDim = 32;
constexpr uint32_t kBos = 1022u;   // rust/src/main.rs:214

// Exact integer arithmetic on the FP32 pipes.  A float in [2^23, 2^24) has spacing 1,
// and a fused multiply-add rounds its exact result once, to nearest with ties to even,
// which is the reference's round-half-to-even shift (rust/src/primitives.rs:18-73).
// With the bias M1 = 1.5 * 2^23 (bits kM1Bits), an integer |x| < 2^22 is the float
// M1 + x, whose bits are kM1Bits + x, and fma(M1 + x, m, M1 - M1 * m) = M1 + rne(x * m)
// whenever m and M1 - M1 * m are exact floats and |x * m| < 2^22.  The low byte of
// the bits of M1 + y is y mod 256, so small results pack into int8 lanes directly.
constexpr uint32_t kM1Bits = 0x4B400000u;   // 12582912.0f
constexpr float kM1 = 12582912.0f;

// SMs of the current device (cached per device): persistent grids are sized by it
inline int sm_count() {
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

// Programmatic dependent launch.  A kernel launched with the PDL attribute may be
// scheduled while the previous kernel of its stream is still running: pdl_wait()
// blocks until that kernel has completed and its memory writes are visible (for a
// normal launch it returns at once), so every kernel that launch_k may launch with
// the attribute calls it before its first access to memory that another kernel
// writes.  pdl_trigger() lets the next kernel of the stream begin to launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// launch_k: a kernel launch that carries the PDL attribute while g_pdl_launch is set
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (g_pdl_launch) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// primitives.rs:9-11
__device__ __forceinline__ int clamp127(int x) { return min(127, max(-127, x)); }

// primitives.rs:18-42.  Round-half-even is symmetric, so flooring the signed
// value and rounding the remainder equals the reference's sign-magnitude form.
__device__ __forceinline__ int sra_rne32(int v, int sh) {
    if (sh == 0) return v;
    int q = v >> sh;
    uint32_t r = (uint32_t)v & ((1u << sh) - 1u);
    uint32_t half = 1u << (sh - 1);
    q += (r > half) | ((r == half) & (q & 1));
    return q;
}

// The RoPE roundings (attention.rs:29-83) of v = x*cos -/+ y*sin, |v| <= 2^23 (int8 x, y;
// int16 cos, sin): clamp127(rne(v / 2^15)) for keys and clamp127(rne(rne(v / 2^15) / 2))
// for queries, in FP32.  v converts exactly; with M1 = 1.5 * 2^23, fma(v, 2^-15, M1) is
// M1 + v / 2^15 (|v / 2^15| <= 256) rounded once to spacing 1, ties to even: M1 +
// rne(v / 2^15), and fma(that, 1/2, M1/2) = M1 + rne(rne(v / 2^15) / 2) likewise; the
// bias comes off inside the clamp.  Checked against the integer forms for every v in
// [-2^23, 2^23] (tests/rope_round_fp32.c).
__device__ __forceinline__ int rope_k_round(int v) {
    const int b = __float_as_int(__fmaf_rn(__int2float_rn(v), 1.0f / 32768.0f, 12582912.0f));
    return min(__viaddmax_s32(b, -(int)kM1Bits, -127), 127);
}
__device__ __forceinline__ int rope_q_round(int v) {
    const float r1 = __fmaf_rn(__int2float_rn(v), 1.0f / 32768.0f, 12582912.0f);
    const int b = __float_as_int(__fmaf_rn(r1, 0.5f, 6291456.0f));
    return min(__viaddmax_s32(b, -(int)kM1Bits, -127), 127);
}

// primitives.rs:49-73 (result saturated to the int32 range)
__device__ __forceinline__ int sra_rne64_to32(long long v, int sh) {
    long long q = v;
    if (sh > 0) {
        q = v >> sh;
        unsigned long long r = (unsigned long long)v & ((1ull << sh) - 1ull);
        unsigned long long half = 1ull << (sh - 1);
        q += (r > half) | ((r == half) & (q & 1));
    }
    q = q < -2147483648ll ? -2147483648ll : q;
    q = q > 2147483647ll ? 2147483647ll : q;
    return (int)q;
}

// model.rs:280-300 -- requantise an int32 accumulator to int8
__device__ __forceinline__ int requant(int acc, int mult, int shift) {
    long long p = (long long)acc * (long long)mult;
    if (shift <= 0) {
        p = p < -127 ? -127 : (p > 127 ? 127 : p);
        return (int)p;
    }
    return clamp127(sra_rne64_to32(p, shift));
}

// lut.rs:213-235 == softmax_cdf.rs:55-77: Q16 weight of a non-positive difference
__device__ __forceinline__ uint32_t exp_q16(int neg_x, const uint16_t *lut, uint32_t coef) {
    if (neg_x >= 0) return 65535u;
    uint32_t neg = 0u - (uint32_t)neg_x;
    uint32_t t256 = (uint32_t)(((unsigned long long)neg * coef + (1ull << 23)) >> 24);
    uint32_t ip = t256 >> 8;
    if (ip >= 31) return 1u;
    uint32_t out = (((1u << 16) >> ip) * (uint32_t)lut[t256 & 255u] + 0x8000u) >> 16;
    return min(65535u, max(1u, out));
}

// exp_q16 rewritten without the multiply by 65536 >> ip: for ip >= 1,
// ((2^16 >> ip) * l + 2^15) >> 16 == (l + 2^(ip-1)) >> ip (both are l / 2^ip
// rounded half up, and 0 for ip > 16).  Same values as exp_q16 for every input.
__device__ __forceinline__ uint32_t exp_q16_shift(int neg_x, const uint16_t *lut, uint32_t coef) {
    if (neg_x >= 0) return 65535u;
    const uint32_t neg = 0u - (uint32_t)neg_x;
    const uint32_t t256 = (uint32_t)(((unsigned long long)neg * coef + (1ull << 23)) >> 24);
    const uint32_t ip = t256 >> 8;
    if (ip >= 31) return 1u;
    const uint32_t out = ((uint32_t)lut[t256 & 255u] + ((1u << ip) >> 1)) >> ip;
    return min(65535u, max(1u, out));
}

// 1 + floor(e * R / S) (softmax_cdf.rs:113-121) for e < 2^16 and S < 2^26, with
// a = R / S and F a 32-bit fixed-point fraction of b / S (b = R % S) from below:
// F <= b * 2^32 / S < F + 2818.  Then q0 = hi(e * F) is floor(e * b / S) or one
// less, and the remainder e*R - (e*a + q0)*S, which lies in [0, 2S) and so is
// exact in wrapping 32-bit arithmetic, decides.  F comes from the correctly
// rounded float b / S: b, S and the quotient each round with relative error
// <= 2^-24, so bs * 2^32 is within 770 of b * 2^32 / S, and 2048 less is below it.
struct FreqDiv {
    uint32_t R, S, a, F;
};
__device__ __forceinline__ FreqDiv make_freq_div(uint32_t R, uint32_t S) {
    FreqDiv d;
    d.R = R;
    d.S = S;
    d.a = R / S;
    const float bs = __fdiv_rn(__uint2float_rn(R - d.a * S), __uint2float_rn(S));
    const float p = __fmul_rn(bs, 4294967296.0f);
    const uint32_t fe = p >= 4294967296.0f ? 0xFFFFFFFFu : __float2uint_rz(p);
    d.F = fe > 2048u ? fe - 2048u : 0u;
    return d;
}
__device__ __forceinline__ uint32_t freq_of(uint32_t e, const FreqDiv &d) {
    const uint32_t q = e * d.a + __umulhi(e, d.F);
    const uint32_t r = e * d.R - q * d.S;
    return q + (r >= d.S ? 2u : 1u);
}

// primitives.rs:192-213 -- floor(sqrt(x)), which the reference computes with the
// restoring digit-by-digit method.  Here: the correctly rounded float square root
// of the correctly rounded float of x is within one of floor(sqrt(x)) for every
// 32-bit x, and one step in each direction makes it exact (checked against the
// restoring method for all 2^32 inputs).
__device__ __forceinline__ uint32_t isqrt32(uint32_t x) {
    uint32_t r = (uint32_t)__fsqrt_rn(__uint2float_rn(x));
    if ((unsigned long long)r * r > x) r--;
    else if ((unsigned long long)(r + 1) * (r + 1) <= x) r++;
    return r;
}

__device__ __forceinline__ uint32_t udiv_rne32(uint32_t n, uint32_t d) {
    if (d == 0) return 0;
    uint32_t q = n / d, r = n - q * d, tr = r << 1;
    if (tr > d) return q + 1;
    if (tr == d) return q + (q & 1u);
    return q;
}

// rmsnorm.rs:14-30 with mean_sq = floor(sum_sq / d) + eps (rmsnorm.rs:53-58)
__device__ __forceinline__ int inv_rms_q15(uint32_t sum_sq, int d, int eps) {
    int mean_sq = (int)(sum_sq / (uint32_t)d) + eps;
    uint32_t ms = mean_sq > 0 ? (uint32_t)mean_sq : 1u;
    uint32_t inv = udiv_rne32(8388608u, isqrt32(ms << 16));
    return (int)min(32768u, max(1u, inv));
}

// primitives.rs:163-185; the final `(q as i32) * sign` wraps like Rust release
__device__ __forceinline__ int div_rne_s32_u64(int num, unsigned long long den) {
    if (den == 0) return 0;
    bool neg = num < 0;
    uint32_t an = neg ? 0u - (uint32_t)num : (uint32_t)num;
    unsigned long long q, r;
    if (den <= 0xFFFFFFFFull) {
        uint32_t d32 = (uint32_t)den;
        uint32_t q32 = an / d32;
        q = q32;
        r = an - q32 * d32;
    } else {
        q = 0;
        r = an;
    }
    unsigned long long tr = r << 1;
    if (tr > den) q += 1;
    else if (tr == den) q += (q & 1ull);
    uint32_t q32 = (uint32_t)q;
    return (int)(neg ? 0u - q32 : q32);
}

// div_rne_s32_u64 for many numerators over one denominator.  A denominator of
// 2^32 or more gives 0 for every |num| <= 2^31 (the doubled remainder never
// exceeds it, and a tie rounds to the even 0).  Below that, inv = floor((2^32-1)/d)
// makes umulhi(|num|, inv) at most one below floor(|num| / d) for |num| <= 2^31,
// so one correction step gives the exact quotient and remainder.
struct RneDiv {
    uint32_t d, inv;
};

__device__ __forceinline__ RneDiv make_rne_div(unsigned long long den) {
    RneDiv v;
    v.d = den > 0xFFFFFFFFull ? 0u : (uint32_t)den;   // 0: every quotient is 0
    v.inv = v.d ? 0xFFFFFFFFu / v.d : 0u;
    return v;
}

__device__ __forceinline__ int div_rne_s32_by(int num, RneDiv v) {
    if (v.d == 0u) return 0;
    const bool neg = num < 0;
    const uint32_t an = neg ? 0u - (uint32_t)num : (uint32_t)num;
    uint32_t q = __umulhi(an, v.inv);
    uint32_t r = an - q * v.d;
    if (r >= v.d) { q += 1u; r -= v.d; }
    const uint32_t half = v.d - r;   // 2r > d  <=>  r > d - r
    if (r > half) q += 1u;
    else if (r == half) q += q & 1u;
    return (int)(neg ? 0u - q : q);
}

// clamp127(rne(x / d)) for d >= 1 (d < 2^32), with rcp = the correctly rounded float
// of 1 / float(d): the float product of float(x) and rcp is within a relative 2^-22 of
// x / d, so within 2^-15 wherever the quotient is below 128 in magnitude (beyond it
// the clamp decides).  Unless it lies within 2^-14 of a half, its nearest integer is
// then the nearest integer of x / d (ties cannot be that close to a non-tie: they are
// 1 / (2d) >= 2^-33 apart); the rest take the exact integer division.
__device__ __forceinline__ int div_rne_clamp127(int x, uint32_t d, float rcp) {
    const float qf = __fmul_rn(__int2float_rn(x), rcp);
    const float kf = rintf(qf);
    int q;
    if (fabsf(__fsub_rn(qf, kf)) <= 0.5f - 1.0f / 16384.0f) q = __float2int_rn(kf);
    else q = div_rne_s32_by(x, make_rne_div(d));
    return clamp127(q);
}

// floor(a / d) for a < 2^62 and d > 0 given inv = floor((2^64 - 1) / d):
// the estimate umulhi(a, inv) is at most one below the quotient.
__device__ __forceinline__ unsigned long long udiv_by_inv(unsigned long long a,
                                                          unsigned long long d,
                                                          unsigned long long inv) {
    unsigned long long q = __umul64hi(a, inv);
    unsigned long long r = a - q * d;
    if (r >= d) q += 1;
    return q;
}

__device__ __forceinline__ int sext8(uint32_t w, int byte) {
    return (int)(int8_t)((w >> (8 * byte)) & 0xFFu);
}

// V tile of 32 keys x 64 dims (2 KB) in the attention kernels' streamed and decode
// layouts, lane-major: the P.V A fragment of lane l = 4g + t (mma m16n8k32, V^T as A)
// is 16 words va[mi][k] = 4 bytes of keys 8t + 4(k >> 1) .. +3 at dim
// 16 mi + g + 8 (k & 1), stored as the 16-byte chunk mi at chunk position
// mi ^ ((l >> 1) & 3) of the lane's 64 bytes, so a lane loads its fragments with four
// 16-byte loads and the eight lanes of each load phase hit eight bank groups.
// Returns the byte of (key, dim) in the tile.
__device__ __forceinline__ int vt_byte(int key, int dim) {
    const int t = key >> 3, kb = (key >> 2) & 1, b = key & 3;
    const int mi = dim >> 4, g = dim & 7, h = (dim >> 3) & 1;
    const int lane = 4 * g + t;
    return 64 * lane + 16 * (mi ^ ((lane >> 1) & 3)) + 4 * (2 * kb + h) + b;
}

}  // namespace czg
