"""Known-answer tests of the reference's Rust test modules, run against the C oracle.

Each test cites the reference test it restates (rust/src/<file>:<lines>).
"""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def L(oracle_mod):
    return oracle_mod.lib()


def test_sra_rne_s32(L):
    # primitives.rs:306-333
    f = L.czo_sra_rne_s32
    assert [f(100, 1), f(64, 2), f(-100, 1)] == [50, 16, -50]
    assert [f(3, 1), f(5, 1), f(7, 1)] == [2, 2, 4]
    assert [f(-3, 1), f(-5, 1), f(-7, 1)] == [-2, -2, -4]
    assert [f(5, 2), f(7, 2)] == [1, 2]


def test_isqrt(L):
    # primitives.rs:336-345
    f = L.czo_isqrt32
    cases = {0: 0, 1: 1, 4: 2, 9: 3, 15: 3, 16: 4, 65536: 256, 0xFFFFFFFF: 65535}
    for x, want in cases.items():
        assert f(x) == want


def test_udiv_rne(L):
    # primitives.rs:348-363
    f = L.czo_udiv_rne_u32
    assert [f(10, 2), f(12, 4)] == [5, 3]
    assert [f(3, 2), f(5, 2), f(7, 2)] == [2, 2, 4]
    assert f(7, 4) == 2


def test_clamp_i8(L):
    # primitives.rs:366-376
    f = L.czo_clamp_i8
    for x, want in [(0, 0), (127, 127), (128, 127), (-127, -127), (-128, -127), (-129, -127),
                    (1000, 127), (-1000, -127)]:
        assert f(x) == want


def test_reglu(oracle_mod):
    # reglu.rs:62-99
    L = oracle_mod.lib()
    P = oracle_mod.ptr

    def run(x, dff):
        x = np.array(x, dtype=np.int8)
        out = np.zeros(dff, dtype=np.int8)
        L.czo_reglu(P(x), dff, P(out))
        return out.tolist()

    assert run([-64, 100], 1) == [0]
    assert run([64, 64], 1) == [32]
    assert run([32, 64], 1) == [16]
    assert run([32, 2], 1) == [0]
    assert run([96, 2], 1) == [2]


def test_linear(oracle_mod):
    # linear.rs:85-128
    L = oracle_mod.lib()
    P = oracle_mod.ptr

    def lin(x, w, i, o):
        x = np.array(x, dtype=np.int8)
        w = np.array(w, dtype=np.int8)
        y = np.zeros(o, dtype=np.int32)
        L.czo_linear_i8_i32(P(x), P(w), i, o, P(y))
        return y.tolist()

    assert lin([1, 2], [1, 0, 0, 1], 2, 2) == [1, 2]
    assert lin([1, 2, 3], [1, 1, 1], 3, 1) == [6]
    assert lin([-10, 10], [1, 1], 2, 1) == [0]
    assert lin([127] * 64, [127] * 64, 64, 1) == [127 * 127 * 64]


def test_inv_rms(L):
    # rmsnorm.rs:136-148
    f = L.czo_inv_rms_q15
    assert [f(1), f(4), f(16), f(16384)] == [32768, 16384, 8192, 256]


def test_rmsnorm_zero(oracle_mod):
    # rmsnorm.rs:151-160
    L, P = oracle_mod.lib(), oracle_mod.ptr
    x = np.zeros(4, dtype=np.int8)
    w = np.full(4, 127, dtype=np.int8)
    out = np.ones(4, dtype=np.int8)
    L.czo_rmsnorm_i8(P(x), P(w), 4, 1, P(out))
    assert out.tolist() == [0, 0, 0, 0]


def test_requant(oracle_mod):
    # model.rs:502-508
    L, P = oracle_mod.lib(), oracle_mod.ptr
    x = np.array([8192, 4096, -8192], dtype=np.int32)
    out = np.zeros(3, dtype=np.int8)
    L.czo_requant(P(x), 3, 1, 7, P(out))
    assert out.tolist() == [64, 32, -64]


def test_attn_coef(L):
    # attention.rs:330-334; also the CDF constant pinned at
    # python/tests/test_cross_language.py:32-45
    assert L.czo_attn_coef_q24() == int((1.4426950408889634 / 64.0) * (1 << 24) + 0.5)
    assert L.czo_default_coef_q24() == 37819
    assert L.czo_default_target_total(1024) == 1073739776
    assert L.czo_default_target_total(1024) < (1 << 30)


def test_rope_identity_pos0(oracle_mod, shipped_oracle):
    # attention.rs:296-307 (cos = 32767, sin = 0 at position 0)
    L, P = oracle_mod.lib(), oracle_mod.ptr
    t = shipped_oracle.tensors
    x = np.full(64, 64, dtype=np.int8)
    L.czo_rope_k(P(x), P(t["lut.rope_cos"]), P(t["lut.rope_sin"]), 0)
    assert np.all(np.abs(x.astype(int) - 64) <= 1)


def _cdf(oracle_mod, logits, V):
    lut = np.zeros(256, dtype=np.uint16)
    # Exp2LutQ16::new (lut.rs:40-51): round(2^(-i/256) * 65536) clamped to [1, 65535]
    for i in range(256):
        lut[i] = min(65535, max(1, int(np.rint(2.0 ** (-i / 256.0) * 65536.0))))
    L = oracle_mod.lib()
    return oracle_mod.build_cumfreqs(np.array(logits, np.int32), lut, L.czo_default_coef_q24(),
                                     L.czo_default_target_total(V))


def test_cumfreqs_properties(oracle_mod):
    # softmax_cdf.rs:185-248
    L = oracle_mod.lib()
    lg = [100, 50, 25, 10, 5, 0, -5, -10, -25, -50, -100, -200, -300, -400, -500, -1000]
    cum = _cdf(oracle_mod, lg, 16)
    assert cum[15] == L.czo_default_target_total(16)
    assert np.all(np.diff(cum.astype(np.int64)) > 0)
    cum = _cdf(oracle_mod, [10000, -10000, -10000, -10000], 4)
    assert cum[0] >= 1 and np.all(np.diff(cum.astype(np.int64)) >= 1)
    cum = _cdf(oracle_mod, [100, 100, 100, 100], 4)
    assert cum[0] >= cum[1] - cum[0]


def test_coder_roundtrips(oracle_mod):
    # arith_coder.rs:277-348 (uniform cumfreqs, round trips)
    def uni(n):
        return np.arange(1, n + 1, dtype=np.uint32) * 1000

    for n, syms in [(4, [2]), (8, [0, 3, 7, 2, 5, 1]), (8, [i % 8 for i in range(16)])]:
        rows = [uni(n)] * len(syms)
        data = oracle_mod.encode_symbols(rows, syms)
        assert oracle_mod.decode_symbols(data, rows) == syms
