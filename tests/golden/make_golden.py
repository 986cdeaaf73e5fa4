"""Generate golden vectors from the reference's own Python mirror.

Runs only where the reference tree is mounted (read-only, never copied):
    python tests/golden/make_golden.py /path/to/compress-zip
and writes tests/golden/pyref_vectors.npz, which the CPU test suite checks the
C oracle against.

The reference's Python package does not import as shipped (its model module
raises at class creation), so the individual modules on this path are loaded
without the package __init__.  Functions where the Python mirror is known to
differ from the Rust crate are handled as follows:

* udiv_rne_tte_u32 rounds odd-divisor "ties" up in Python
  (python/compress_zip/primitives.py:102-109) but not in Rust
  (rust/src/primitives.rs:88-96).  RMSNorm rows whose mean square reaches such a
  divisor are flagged (``rms_divergent``) instead of being used as vectors;
* the Python attention clips its output to [-128, 127]
  (python/compress_zip/attention.py:409) where Rust clamps to [-127, 127], and
  keeps int64 accumulators; the cases drawn here never overflow i32, and a -128
  output, if any, is recorded so the test can expect -127.

Everything else (ties-to-even shifts, isqrt, both exp functions, RoPE, ReGLU,
build_cumfreqs, the arithmetic coder bytes) is taken from the Python mirror
unchanged.  Inputs come from a seeded numpy generator.
"""
from __future__ import annotations

import importlib
import os
import sys
import types

import numpy as np

SEED = 1234


def load_reference(root: str):
    pkg = types.ModuleType("compress_zip")
    pkg.__path__ = [os.path.join(root, "python", "compress_zip")]
    sys.modules["compress_zip"] = pkg
    mods = {}
    for m in ["primitives", "lut", "rmsnorm", "reglu", "softmax_cdf", "arith_coder", "attention"]:
        mods[m] = importlib.import_module("compress_zip." + m)
    return types.SimpleNamespace(**mods)


def shipped_tables(root: str):
    from safetensors import safe_open

    with safe_open(os.path.join(root, "models", "v001_eng.czm"), "np") as f:
        return {k: f.get_tensor(k) for k in ["lut.exp2", "lut.rope_cos", "lut.rope_sin",
                                               "layers.0.attn.score_mult", "norm.weight",
                                               "layers.0.post_ffn_norm.weight",
                                               "softmax.coef_q24", "softmax.target_total"]}


def main(root: str, out_path: str) -> None:
    R = load_reference(root)
    T = shipped_tables(root)
    rng = np.random.Generator(np.random.PCG64(SEED))
    lut = T["lut.exp2"].astype(np.uint16)
    cos, sin = T["lut.rope_cos"], T["lut.rope_sin"]
    coef = int(T["softmax.coef_q24"])
    total = int(T["softmax.target_total"])
    g = {}

    # --- shifts, isqrt, division -----------------------------------------------------
    v = np.concatenate([rng.integers(-2**31, 2**31, 3000), rng.integers(-4096, 4096, 1000),
                        [0, 1, -1, 3, -3, 5, -5, 7, -7, 2**31 - 1, -2**31 + 1]]).astype(np.int64)
    sh = rng.integers(1, 21, len(v))
    g["sra32_in"], g["sra32_sh"] = v.astype(np.int32), sh.astype(np.uint32)
    g["sra32_out"] = np.array([R.primitives.sra_rne_tte_s32(int(a), int(b))
                               for a, b in zip(v, sh)], dtype=np.int32)
    v64 = rng.integers(-2**45, 2**45, 3000, dtype=np.int64)
    sh64 = rng.integers(1, 33, len(v64))
    g["sra64_in"], g["sra64_sh"] = v64, sh64.astype(np.uint32)
    g["sra64_out"] = np.array([R.primitives.sra_rne_tte_s64_to_s32(int(a), int(b))
                               for a, b in zip(v64, sh64)], dtype=np.int32)
    xs = np.concatenate([rng.integers(0, 2**32, 3000), np.arange(0, 300),
                         [0xFFFFFFFF, 65536, 65535, 1 << 30]]).astype(np.uint64)
    g["isqrt_in"] = xs.astype(np.uint32)
    g["isqrt_out"] = np.array([R.primitives.isqrt32_restoring(int(x)) for x in xs], dtype=np.uint32)
    num = rng.integers(-2**31 + 1, 2**31, 3000)
    den = rng.integers(1, 2**26, 3000)
    den[:500] = 2 * np.abs(num[:500]) // 5 + 1
    g["div_num"], g["div_den"] = num.astype(np.int32), den.astype(np.uint64)
    g["div_out"] = np.array([R.primitives.div_rne_tte_s64_to_s32(int(a), int(b))
                             for a, b in zip(num, den)], dtype=np.int32)

    # --- exp functions ----------------------------------------------------------------
    diffs = np.concatenate([-rng.integers(0, 2**21, 4000), -np.arange(0, 2000),
                            [0, -1, -2**31 + 1]]).astype(np.int64)
    g["exp_diff"] = diffs.astype(np.int32)
    g["exp_cdf_out"] = np.array([R.softmax_cdf.exp_q16_from_diff_acc(int(d), lut, coef)
                                 for d in diffs], dtype=np.uint16)
    g["exp_attn_out"] = np.array([R.attention.exp_q16_from_attn_diff(int(d), lut)
                                  for d in diffs], dtype=np.uint16)

    # --- RMSNorm ----------------------------------------------------------------------
    d = 384
    w = T["layers.0.post_ffn_norm.weight"].astype(np.int8)
    rows, div_flags = [], []
    for i in range(400):
        scale = [1, 3, 10, 40, 127][i % 5]
        rows.append(np.clip(rng.integers(-scale, scale + 1, d), -127, 127).astype(np.int8))
    rows.append(np.zeros(d, np.int8))
    rows.append(np.full(d, 127, np.int8))
    rows.append(np.full(d, -127, np.int8))
    X = np.stack(rows)
    Y = np.stack([R.rmsnorm.rmsnorm_i8(x, w, 1) for x in X])
    for x in X:
        ms = int(np.sum(x.astype(np.int64) ** 2)) // d + 1
        s = R.primitives.isqrt32_restoring(max(ms, 1) << 16)
        q, r = divmod(8388608, s)
        div_flags.append(bool(s % 2 == 1 and r == s // 2))
    g["rms_x"], g["rms_w"], g["rms_out"] = X, w, Y.astype(np.int8)
    g["rms_divergent"] = np.array(div_flags)
    ms_all = np.arange(1, 16131)
    g["inv_rms_ms"] = ms_all.astype(np.int32)
    g["inv_rms_py"] = np.array([R.rmsnorm.compute_inv_rms_q15_from_mean_sq(int(m))
                                for m in ms_all], dtype=np.int32)

    # --- ReGLU, RoPE ------------------------------------------------------------------
    gate = rng.integers(-127, 128, 5000).astype(np.int8)
    val = rng.integers(-127, 128, 5000).astype(np.int8)
    g["reglu_gate"], g["reglu_val"] = gate, val
    g["reglu_out"] = R.reglu.reglu_i8(gate, val).astype(np.int8)
    rx = rng.integers(-127, 128, (300, 64)).astype(np.int8)
    rpos = rng.integers(0, cos.shape[0], 300)
    g["rope_x"], g["rope_pos"] = rx, rpos.astype(np.int32)
    g["rope_k_out"] = np.stack([R.attention.apply_rope_i8(x, int(p), cos, sin)
                                for x, p in zip(rx, rpos)]).astype(np.int8)
    g["rope_q_out"] = np.stack([R.attention.apply_rope_q_i8(x, int(p), cos, sin)
                                for x, p in zip(rx, rpos)]).astype(np.int8)

    # --- attention sequences (one head, the reference KV-cache path) ------------------
    sm_all = T["layers.0.attn.score_mult"].astype(np.int64)
    n = 48
    seqs_q, seqs_k, seqs_v, seqs_sm, seqs_out = [], [], [], [], []
    for s_i in range(12):
        amp = [8, 30, 60, 127][s_i % 4]
        q = rng.integers(-amp, amp + 1, (n, 64)).astype(np.int8)
        k = rng.integers(-amp, amp + 1, (n, 64)).astype(np.int8)
        vv = rng.integers(-127, 128, (n, 64)).astype(np.int8)
        smv = int(sm_all[s_i % len(sm_all)])
        cache = R.attention.KVCache.create(max_seq_len=n, head_dim=64)
        outs = [R.attention.gqa_attention_mqa_i8(q[t], k[t], vv[t], t, cache, lut, cos, sin, smv)
                for t in range(n)]
        seqs_q.append(q); seqs_k.append(k); seqs_v.append(vv); seqs_sm.append(smv)
        seqs_out.append(np.stack(outs).astype(np.int16))
    g["attn_q"], g["attn_k"], g["attn_v"] = np.stack(seqs_q), np.stack(seqs_k), np.stack(seqs_v)
    g["attn_sm"], g["attn_out"] = np.array(seqs_sm, np.int32), np.stack(seqs_out)

    # --- softmax -> CDF (V = 1024 with the shipped LUT and constants) -------------------
    logit_rows = []
    for i in range(24):
        amp = [100, 5000, 50000, 400000][i % 4]
        logit_rows.append(rng.integers(-amp, amp + 1, 1024))
    tie = rng.integers(-3000, 3000, 1024)
    tie[[7, 100, 900]] = 5000
    logit_rows += [tie, np.zeros(1024, np.int64), np.arange(1024) * 997 - 500000]
    L = np.stack(logit_rows).astype(np.int32)
    g["cdf_logits"] = L
    g["cdf_cum"] = np.stack([R.softmax_cdf.build_cumfreqs(l, 1024, lut, coef, total)[0]
                             for l in L]).astype(np.uint32)
    g["cdf_coef"], g["cdf_total"] = np.uint32(coef), np.uint32(total)
    g["lut"] = lut

    # --- arithmetic coder bytes ---------------------------------------------------------
    # CDFs over V = 64 built by the reference from random logits (several peaks),
    # plus the uniform CDFs of the Rust tests (rust/src/arith_coder.rs:271-275).
    Vc = 64
    tot_c = int(R.softmax_cdf.compute_target_total(Vc))
    streams = []
    for s_i in range(8):
        nsym = [1, 5, 60, 400, 400, 400, 400, 700][s_i]
        amp = [0, 2000, 20000, 200000, 2000000, 50000, 800, 30000][s_i]
        cums, syms = [], []
        for _ in range(nsym):
            lg = rng.integers(-amp, amp + 1, Vc).astype(np.int32)
            cum, _t = R.softmax_cdf.build_cumfreqs(lg, Vc, lut, coef, tot_c)
            cums.append(cum)
            if s_i == 5:   # mostly the least likely symbol: long bit runs
                syms.append(int(np.argmin(np.diff(np.concatenate([[0], cum])))))
            elif s_i == 6:  # mostly the most likely symbol: pending-bit (E3) runs
                syms.append(int(np.argmax(np.diff(np.concatenate([[0], cum])))))
            else:
                syms.append(int(rng.integers(0, Vc)))
        enc = R.arith_coder.ArithEncoder()
        for c, s in zip(cums, syms):
            enc.encode_symbol(c, s, int(c[-1]))
        streams.append((np.stack(cums).astype(np.uint32), np.array(syms, np.int32), enc.finish()))
    for nsym_u, V_u in [(1, 4), (6, 8), (16, 8)]:
        cum = (np.arange(1, V_u + 1) * 1000).astype(np.uint32)
        syms = [int(x) for x in rng.integers(0, V_u, nsym_u)]
        enc = R.arith_coder.ArithEncoder()
        for s in syms:
            enc.encode_symbol(cum, s, int(cum[-1]))
        streams.append((np.tile(cum, (nsym_u, 1)), np.array(syms, np.int32), enc.finish()))
    for i, (c, s, b) in enumerate(streams):
        g[f"coder{i}_cum"], g[f"coder{i}_sym"] = c, s
        g[f"coder{i}_bytes"] = np.frombuffer(b, dtype=np.uint8)
    g["coder_n"] = np.int32(len(streams))
    np.savez_compressed(out_path, **g)
    print(f"wrote {out_path}: {len(g)} arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <compress-zip checkout>")
    root = sys.argv[1]
    here = os.path.dirname(os.path.abspath(__file__))
    main(root, os.path.join(here, "pyref_vectors.npz"))
