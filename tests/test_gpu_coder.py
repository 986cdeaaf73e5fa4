"""The compress path's arithmetic encoder on crafted coder intervals.

The GPU encoder (k_encode) renormalises in closed form: all agreeing top bits of
low and high leave at once, then all straddle (E3) steps at once, and a pending
run that does not fit one 32-bit push leaves in pieces.  The reference
(rust/src/arith_coder.rs:80-130) loops bit by bit.  Real text almost never
reaches three branches of the closed form -- an interval that collapses to one
value (32 agreeing bits), 31 straddle steps in one symbol, and pending runs of
more than 32 bits -- so these tests feed interval sequences built to reach them
(tests/coder_cases.py), plus random intervals of every width, to the encoder
through czg_debug_encode_intervals and compare the bytes with the CPU oracle's
encoder.  The allocation-free encoder gets the same intervals.
"""
import ctypes as C

import numpy as np
import pytest

import coder_cases as cc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine(shipped_path):
    from compress_zip_b200.engine import Engine

    eng = Engine.from_file(shipped_path, 0)
    yield eng
    eng.close()


def _packed(seqs):
    lohi = np.array([p for s in seqs for p in s], dtype=np.uint32).reshape(-1, 2)
    starts = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.uint64)
    return lohi, starts


@pytest.mark.parametrize("kind", ["crafted", "random"])
def test_encoder_matches_oracle_on_crafted_intervals(engine, oracle_mod, kind):
    total = engine.info["target_total"]
    seqs = cc.crafted_sequences(total) if kind == "crafted" else cc.random_sequences(total)
    cov = cc.branch_counts(seqs, total)
    if kind == "crafted":   # the sequences do reach the rare branches
        assert cov["all_32_agree"] > 0 and cov["straddle_31"] > 0 and cov["pending_over_64"] > 0, cov
    lohi, starts = _packed(seqs)
    got = engine.debug_encode_intervals(lohi, starts)
    want = [oracle_mod.encode_intervals(s, total) for s in seqs]
    assert len(got) == len(want)
    for i, (a, b) in enumerate(zip(got, want)):
        assert a == b, f"sequence {i} differs ({kind})"


def test_static_encoder_on_crafted_intervals(engine, oracle_mod):
    """The allocation-free encoder (bit-loop renormalisation) on the same intervals."""
    import torch

    from compress_zip_b200 import engine as E

    total = engine.info["target_total"]
    seqs = cc.crafted_sequences(total, seed=3)
    lohi, starts = _packed(seqs)
    lens = np.diff(starts).astype(np.uint32)
    d_lohi = torch.from_numpy(lohi.view(np.int32).reshape(-1)).cuda()
    d_len = torch.from_numpy(lens.view(np.int32)).cuda()
    cap = 4 * len(lohi) + 8 * len(lens)
    d_out = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    d_out_lens = torch.zeros(len(lens), dtype=torch.int32, device="cuda")
    nbytes = C.c_uint64(0)
    st = E.lib().czg_encode_intervals_static(d_lohi.data_ptr(), d_len.data_ptr(), len(lens), len(lohi), total,
                                             d_out.data_ptr(), cap, d_out_lens.data_ptr(), C.byref(nbytes),
                                             C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    want = [oracle_mod.encode_intervals(s, total) for s in seqs]
    assert nbytes.value == sum(len(w) for w in want)
    assert d_out[: nbytes.value].cpu().numpy().tobytes() == b"".join(want)
    assert list(d_out_lens.cpu().numpy().view(np.uint32)) == [len(w) for w in want]
