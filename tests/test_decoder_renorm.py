"""The batched decoder renormalises in closed form (decode.cu, dec_narrow): n1 =
clz(low ^ high) E1/E2 shifts, then the run of E3 steps read off low & ~high, with
the chunk bits from one 64-bit window.  This CPU test restates those formulas in C
and checks them against the reference's bit-at-a-time loop
(rust/src/arith_coder.rs:244-264) on 4 M random and edge states, garbage ones
included, with reads past the chunk's end giving 0."""
import os
import shutil
import subprocess

import pytest


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_closed_form_renormalisation_matches_loop(tmp_path):
    src = os.path.join(os.path.dirname(os.path.abspath(__file__)), "renorm_closed_form.c")
    exe = tmp_path / "renorm_closed_form"
    subprocess.run(["gcc", "-O2", "-std=c11", src, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 bad" in out.stdout
