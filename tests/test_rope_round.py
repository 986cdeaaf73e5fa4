"""The kernels round the RoPE products in FP32 (rope_k_round and rope_q_round in
compress-zip_b200/csrc/common.cuh).  This CPU test restates both in C with fmaf and
compares them with the integer round-half-even shifts (rust/src/primitives.rs:18-42,
as attention.rs:29-83 applies them) for every reachable product v in [-2^23, 2^23]."""
import os
import shutil
import subprocess

import pytest


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_fp32_rope_rounding_matches_integer_shifts(tmp_path):
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rope_round_fp32.c")
    exe = tmp_path / "rope_round_fp32"
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", src, "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "key 0 bad, query 0 bad" in out.stdout
