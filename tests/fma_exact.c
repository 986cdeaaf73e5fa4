// fma_exact.c -- exhaustive host check of the FP32 score and exp-index formulas of
// attention_mma.cu (score_flt, t256_flt) against the integer arithmetic of the reference
// (rust/src/attention.rs:236-245, rust/src/lut.rs:213-235).  C fmaf is the IEEE fused
// multiply-add the device __fmaf_rn computes.  Exit status 0: every case matches.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
static int32_t sra_rne32(int32_t v, int sh) {  // round half to even
    int64_t q = (int64_t)v >> sh, r = (int64_t)v - (q << sh), h = 1ll << (sh - 1);
    if (r > h || (r == h && (q & 1))) q++;
    return (int32_t)q;
}
static int32_t sra_rne64(int64_t v, int sh) {
    int64_t q = v >> sh, r = v - (q << sh), h = 1ll << (sh - 1);
    if (r > h || (r == h && (q & 1))) q++;
    return (int32_t)q;
}
static float as_f(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t as_u(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
int main(void) {
    /* every dot product of two int8 64-vectors, for the shipped multipliers and edge ones */
    const float M1 = 12582912.0f;   // 1.5 * 2^23
    int mults[] = {58218, 60859, 59427, 58869, 59627, 58811, 1, -1, 3, -3, 2, 32768, -32768, 32767, 65535, 65536,
                   -60000, 100000, 262143, 262144, 400000, -400000, 524287, -524287, 12345, 77777, 131071, -131073,
                   4097, 8191, 17, -99999};
    int nm = sizeof(mults) / sizeof(mults[0]);
    long bad = 0, tot = 0;
    const int DMAX = 64 * 127 * 127;   // |dot| bound of two int8 64-vectors
    for (int mi = 0; mi < nm; mi++) {
        int mult = mults[mi];
        float mf = (float)mult / 32768.0f;
        float c2 = (float)(384 * (32768 - mult));
        if ((double)c2 != 384.0 * (32768.0 - mult)) { printf("c2 inexact for %d\n", mult); return 1; }
        for (int dot = -DMAX; dot <= DMAX; dot++) {
            int32_t du = sra_rne32(dot, 2);
            int32_t ref = sra_rne64((int64_t)du * mult, 15);
            float db = as_f(0x4B400000u + (uint32_t)dot);
            float ub = fmaf(db, 0.25f, 9437184.0f);
            float sb = fmaf(ub, mf, c2);
            int32_t got = (int32_t)(as_u(sb) - 0x4B400000u);
            tot++;
            if (got != ref) { if (bad < 5) printf("mult %d dot %d ref %d got %d\n", mult, dot, ref, got); bad++; }
        }
    }
    printf("scores: %ld checked, %ld bad\n", tot, bad);
    // exp index: t256 = (neg * 378194 + 2^23) >> 24 for neg in [0, 2^23), clamped at 4096
    const float c = 378194.0f / 16777216.0f;
    if ((double)c * 16777216.0 != 378194.0) { printf("c inexact\n"); return 1; }
    long bad2 = 0;
    for (int64_t neg = 0; neg < (1 << 23); neg++) {
        int64_t ref = (neg * 378194 + (1 << 23)) >> 24;
        if (ref > 4096) ref = 4096;
        float nf = (float)neg;   // exact
        float tb = fmaf(nf, c, M1);
        int64_t got = (int64_t)as_u(tb) - 0x4B400000;
        if (got > 4096) got = 4096;
        if (got != ref) { if (bad2 < 5) printf("neg %lld ref %lld got %lld\n", (long long)neg, (long long)ref, (long long)got); bad2++; }
    }
    printf("exp index: %d checked, %ld bad\n", 1 << 23, bad2);
    return bad || bad2;
}
