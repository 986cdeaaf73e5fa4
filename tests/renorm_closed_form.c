// renorm_closed_form.c -- host check of the decoder's closed-form renormalisation
// (decode.cu, dec_narrow) against the bit-at-a-time loop of the reference decoder
// (rust/src/arith_coder.rs:244-264) on random and edge states, garbage ones included
// (low > high, code outside [low, high]), and against the 64-bit window of the chunk
// bits (decode.cu, window_byte / window) with reads past the end giving 0.
// Exit status 0 and "0 bad": every case matches.
#include <stdint.h>
#include <stdio.h>

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static uint64_t next(void) {
    rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17;
    return rng;
}
static int clz32(uint32_t x) { return x ? __builtin_clz(x) : 32; }

static uint32_t read_bit(const uint8_t *d, uint64_t len, uint64_t bit) {
    const uint64_t byte = bit >> 3;
    if (byte >= len) return 0;
    return (d[byte] >> (7 - (bit & 7))) & 1u;
}

// the device window: nine bytes from the byte of `bit`, MSB first, shifted by bit & 7
static uint64_t window64(const uint8_t *d, uint64_t len, uint64_t bit) {
    uint32_t b[9];
    for (int i = 0; i < 9; i++) b[i] = (bit >> 3) + i < len ? d[(bit >> 3) + i] : 0;
    uint32_t hi = 0, lo = 0;
    for (int i = 0; i < 4; i++) hi |= b[i] << (24 - 8 * i);
    for (int i = 4; i < 8; i++) lo |= b[i] << (56 - 8 * i);
    uint64_t w = ((uint64_t)hi << 32) | lo;
    int off = (int)(bit & 7);
    return off ? (w << off) | (b[8] >> (8 - off)) : w;
}

int main(void) {
    uint8_t data[64];
    long bad = 0, tot = 0, e3 = 0, e3long = 0;
    for (long it = 0; it < 4000000; it++) {
        for (int i = 0; i < 64; i++) data[i] = (uint8_t)next();
        const uint64_t len = next() % 65;
        const uint64_t bit0 = next() % (8 * 64);
        uint32_t low = (uint32_t)next(), high = (uint32_t)next(), code = (uint32_t)next();
        switch (it % 6) {   // bias toward long runs of both kinds
            case 0: high = low; break;
            case 1: high = low | (uint32_t)(next() & 0xFF); break;
            case 2: {   // an E3 run of k steps: low = 01 1..1 x, high = 10 0..0 y
                const int k = (int)(next() % 31);
                const uint32_t run = k ? (0xFFFFFFFFu << (32 - k)) >> 2 : 0u;   // bits 29..30-k
                const uint32_t tail = k < 30 ? ((uint32_t)next() & ((1u << (30 - k)) - 1u)) : 0u;
                low = 0x40000000u | run | tail;
                high = 0x80000000u | (k < 30 ? ((uint32_t)next() & ((1u << (30 - k)) - 1u)) : 0u);
                break;
            }
            case 3: low = 0x7FFFFFFFu; high = 0x80000000u; break;
            default: break;
        }
        // the loop (64-bit as the reference)
        const uint64_t HALF = 1ull << 31, QUARTER = 1ull << 30, MASK = 0xFFFFFFFFull;
        uint64_t L = low, H = high, C = code, bit = bit0;
        for (;;) {
            if (((L ^ H) & HALF) == 0) {
                L = (L << 1) & MASK;
                H = ((H << 1) & MASK) | 1ull;
                C = ((C << 1) & MASK) | read_bit(data, len, bit++);
            } else if ((L & ~H & QUARTER) != 0) {
                L = ((L << 1) ^ HALF) & MASK;
                H = (((H ^ HALF) << 1) | HALF | 1ull) & MASK;
                C = (C & HALF) | ((C << 1) & (MASK >> 1)) | read_bit(data, len, bit++);
            } else {
                break;
            }
        }
        // the closed form
        uint64_t win = window64(data, len, bit0);
        uint32_t l = low, h = high, c = code;
        const int n1 = clz32(l ^ h);
        if (n1 > 0) {
            l = (uint32_t)((uint64_t)l << n1);
            h = (uint32_t)(((uint64_t)h << n1) | ((1ull << n1) - 1ull));
            c = (uint32_t)(((uint64_t)c << n1) | (win >> (64 - n1)));
            win <<= n1;
        }
        const int n3 = clz32(~((l & ~h) << 1));
        if (n3 > 0) {
            l = (l << n3) ^ 0x80000000u;
            h = (h << n3) | 0x80000000u | ((1u << n3) - 1u);
            c = (c & 0x80000000u) | ((c << n3) & 0x7FFFFFFFu) | (uint32_t)(win >> (64 - n3));
        }
        tot++;
        e3 += n3 > 0;
        e3long += n3 >= 16;
        if (l != (uint32_t)L || h != (uint32_t)H || c != (uint32_t)C || bit0 + n1 + n3 != bit) {
            if (bad < 5)
                printf("mismatch low %08x high %08x code %08x bit %llu: loop %08x %08x %08x %llu, closed %08x %08x %08x %llu\n",
                       low, high, code, (unsigned long long)bit0, (uint32_t)L, (uint32_t)H, (uint32_t)C,
                       (unsigned long long)bit, l, h, c, (unsigned long long)(bit0 + n1 + n3));
            bad++;
        }
    }
    printf("%ld cases (%ld with E3 steps, %ld with 16 or more), %ld bad\n", tot, e3, e3long, bad);
    return bad != 0;
}
