/* The kernels round the RoPE products (attention.rs:29-83) in FP32 (rope_k_round,
 * rope_q_round in compress-zip_b200/csrc/common.cuh): for v = x*cos -/+ y*sin with
 * int8 x, y and int16 cos, sin (|v| <= 2^23),
 *   key:   clamp127(rne(v / 2^15))           = clamp(fma(v, 2^-15, M1) - M1)
 *   query: clamp127(rne(rne(v / 2^15) / 2))  = clamp(fma(fma(v, 2^-15, M1), 1/2, M1/2) - M1)
 * with M1 = 1.5 * 2^23.  This program compares both with the integer forms of
 * primitives.rs:18-42 (round half to even by shifting) for every v in [-2^23, 2^23]
 * and prints the number of mismatches. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static int sra_rne32(int v, int sh) {
    int q = v >> sh;
    uint32_t r = (uint32_t)v & ((1u << sh) - 1u);
    uint32_t half = 1u << (sh - 1);
    q += (r > half) | ((r == half) & (q & 1));
    return q;
}

static int clamp127(int x) { return x < -127 ? -127 : (x > 127 ? 127 : x); }

static int bits(float f) {
    int b;
    memcpy(&b, &f, 4);
    return b;
}

static const int kM1Bits = 0x4B400000;

static int k_fp32(int v) {
    int b = bits(fmaf((float)v, 1.0f / 32768.0f, 12582912.0f)) - kM1Bits;
    return clamp127(b);
}

static int q_fp32(int v) {
    float r1 = fmaf((float)v, 1.0f / 32768.0f, 12582912.0f);
    int b = bits(fmaf(r1, 0.5f, 6291456.0f)) - kM1Bits;
    return clamp127(b);
}

int main(void) {
    long bad_k = 0, bad_q = 0, n = 0;
    for (int v = -(1 << 23); v <= (1 << 23); v++, n++) {
        if (k_fp32(v) != clamp127(sra_rne32(v, 15))) bad_k++;
        if (q_fp32(v) != clamp127(sra_rne32(sra_rne32(v, 15), 1))) bad_q++;
    }
    printf("%ld values: key %ld bad, query %ld bad\n", n, bad_k, bad_q);
    return (bad_k || bad_q) ? 1 : 0;
}
