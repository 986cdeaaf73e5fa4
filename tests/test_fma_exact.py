"""The attention kernels compute scores and exp-table indices in FP32 when every
|score_mult| < 2^19 (attention_mma.cu, score_flt / t256_flt): a fused multiply-add
rounds once, to nearest with ties to even, and a float in [2^23, 2^24) has spacing 1,
so the biased results are exactly the reference's round-half-to-even integer
arithmetic.  This CPU test checks that claim exhaustively: every dot product of two
int8 64-vectors for a set of multipliers (the shipped ones and edge values up to
2^19 - 1), and every exp index below 2^23, against the integer formulas."""
import os
import shutil
import subprocess

import pytest


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_fp32_score_and_exp_index_exact(tmp_path):
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fma_exact.c")
    exe = tmp_path / "fma_exact"
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", src, "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 bad" in out.stdout
