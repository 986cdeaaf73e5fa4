/* The attention kernels' output division (div_rne_clamp127 in
 * compress-zip_b200/csrc/common.cuh): clamp127(rne(x / d)) (attention.rs:279-284)
 * from the float estimate float(x) * rcp(float(d)), exact unless it lies within
 * 2^-14 of a half, where the integer division decides.  This program restates it
 * with C float arithmetic (round to nearest even, as the device's _rn intrinsics)
 * and compares it with the exact integer form on random, tie and edge cases. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>

static int clamp127(long long x) { return x < -127 ? -127 : (x > 127 ? 127 : (int)x); }

static long long rne_div(long long x, unsigned long long d) {   /* sign-magnitude, ties to even */
    const int neg = x < 0;
    const unsigned long long a = neg ? (unsigned long long)(-x) : (unsigned long long)x;
    unsigned long long q = a / d, r = a % d;
    if (2 * r > d || (2 * r == d && (q & 1))) q++;
    return neg ? -(long long)q : (long long)q;
}

static int fp32_path(int x, uint32_t d, long *fallbacks) {
    const float rcp = 1.0f / (float)d;
    const float qf = (float)x * rcp;
    const float kf = rintf(qf);
    if (fabsf(qf - kf) <= 0.5f - 1.0f / 16384.0f) {
        long long k = (long long)kf;   /* the device saturates; clamped below either way */
        return clamp127(k);
    }
    (*fallbacks)++;
    return clamp127(rne_div(x, d));
}

static uint64_t s = 88172645463325252ull;
static uint64_t rnd(void) { s ^= s << 13; s ^= s >> 7; s ^= s << 17; return s; }

int main(void) {
    long bad = 0, n = 0, fb = 0;
    for (long i = 0; i < 20000000; i++) {
        uint32_t d;
        int x;
        switch (i & 3) {
            case 0: d = (uint32_t)(rnd() >> 32) | 1u; x = (int)(uint32_t)rnd(); break;
            case 1: d = 1u + (uint32_t)(rnd() % 100000u); x = (int)((int64_t)(rnd() % 257) - 128) * (int)(d / 2 + 1) + (int)(rnd() % 7) - 3; break;
            case 2: { d = 2u * (1u + (uint32_t)(rnd() % 1000000u)); long long k = (long long)(rnd() % 300) - 150;
                      x = (int)(k * (long long)d + (long long)(d / 2) * ((rnd() & 1) ? 1 : -1)); break; }   /* exact ties */
            default: d = 1u + (uint32_t)(rnd() >> (32 + (rnd() % 32))); x = (int)((int64_t)(rnd() % 255) - 127) * (int)(d <= 16000000u ? d : 1u); break;
        }
        if (d == 0) d = 1;
        n++;
        if (fp32_path(x, d, &fb) != clamp127(rne_div(x, d))) bad++;
    }
    printf("%ld cases (%ld near a half, divided exactly): %ld bad\n", n, fb, bad);
    return bad ? 1 : 0;
}
