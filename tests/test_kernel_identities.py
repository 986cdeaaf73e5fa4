"""CPU restatements of three integer identities the kernels rely on, checked on
random and edge inputs against the direct forms:

* attention record passes (csrc/attention_mma.cu, seg_ge): with segment bytes
  biased by 0x80, the bytes of segment p are seg >= p and not seg >= p + 1, each
  from one 32-bit subtraction and the bytes' sign bits;
* decoder max and first argmax (csrc/decode.cu, k_cdf_decode_reg<KEY>): for logits
  below 2^26 in magnitude, the largest logit * 32 + (31 - k) of a lane gives its max
  and its first index, and the lowest lane holding the warp max gives the first
  argmax of the row (rust/src/primitives.rs:278-295);
* decoder symbol search (csrc/decode.cu): for code >= low, c = code - low + 1 <=
  range, value = (c * T - 1) // range < X  iff  c * T - 1 < X * range."""
import numpy as np


def _sign_bytes(x):
    return sum((0xFF if (x >> (8 * i + 7)) & 1 else 0) << (8 * i) for i in range(4))


def _seg_ge(segb, p):
    return _sign_bytes((segb - p * 0x01010101) & 0xFFFFFFFF)


def test_segment_masks_by_biased_subtraction():
    rng = np.random.default_rng(5)
    for _ in range(50000):
        segs = np.sort(rng.integers(0, 33, 4))          # non-decreasing, at most 32
        word = sum(int(v) << (8 * i) for i, v in enumerate(segs))
        segb = (word + 0x80808080) & 0xFFFFFFFF
        p = int(rng.integers(0, 33))
        want = sum((0xFF if v == p else 0) << (8 * i) for i, v in enumerate(segs))
        got = _seg_ge(segb, p) & ~_seg_ge(segb, p + 1) & 0xFFFFFFFF
        assert got == want
        if p == 0:
            assert ~_seg_ge(segb, 1) & 0xFFFFFFFF == want


def test_max_and_first_argmax_by_key():
    rng = np.random.default_rng(6)
    E = 32
    for trial in range(3000):
        span = 1 << int(rng.integers(1, 27))
        x = rng.integers(-span + 1, span, size=(32, E)).astype(np.int64)
        if trial % 3 == 0:   # ties, inside and across lanes
            x = rng.integers(-2, 3, size=(32, E)).astype(np.int64) * (span // 4 + 1)
        keys = (x * 32 + (31 - np.arange(E))).max(axis=1)
        lmx = keys >> 5
        mx = lmx.max()
        first = int(np.argmax(lmx == mx))
        am = first * E + 31 - int(keys[first] & 31)
        flat = x.reshape(-1)
        assert mx == flat.max() and am == int(np.argmax(flat == flat.max()))


def test_symbol_search_without_division():
    rng = np.random.default_rng(7)
    T = (1 << 30) - 2048
    for _ in range(100000):
        low = int(rng.integers(0, 1 << 32))
        high = int(rng.integers(low, 1 << 32))
        code = int(rng.integers(low, high + 1))
        rng_ = high - low + 1
        c = code - low + 1
        value = (c * T - 1) // rng_
        X = int(rng.integers(0, 1 << 31))
        if rng.integers(0, 2):
            X = value + int(rng.integers(-1, 2))   # at the boundary
            X = max(X, 0)
        assert (value < X) == (c * T - 1 < X * rng_)
        assert value < (1 << 32)
