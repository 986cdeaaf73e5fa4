"""The attention kernels divide each output sum by the weight sum with a float
estimate and an exact integer fallback within 2^-14 of a half
(div_rne_clamp127 in compress-zip_b200/csrc/common.cuh).  This CPU test restates it
in C and compares it with clamp127(round_half_even(x / d)) (attention.rs:279-284)
on 20 M random, tie and edge cases."""
import os
import shutil
import subprocess

import pytest


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_fp32_output_division_matches_integer(tmp_path):
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "out_div_fp32.c")
    exe = tmp_path / "out_div_fp32"
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", src, "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert ": 0 bad" in out.stdout
