"""Seeded synthetic inputs for the benchmark configurations.

No public corpus is named for this path, so English-like text is generated:
a lexicon of 5,000 distinct lowercase a-z words (lengths uniform in 2..10),
words drawn Zipf(s=1.1) over lexicon rank, sentences of 8-25 words
(capitalised, ending in '.'), paragraphs of 3-7 sentences joined by ' ' and
separated by a blank line, cut or extended to an exact byte count.

``arch2_model`` writes the random-init int8 model of configurations 2 and 4
(d_model 512, 8 layers, 8 query / 2 KV heads, head_dim 64, d_ff 2048) in the
.czm layout the reference loads (rust/src/model.rs:108-274), with RoPE tables
generated as rust/src/lut.rs:97-136 does.
"""
from __future__ import annotations

import math

import numpy as np

from . import czm

LEXICON_SEED = 20240101
LEXICON_SIZE = 5000
ZIPF_S = 1.1

_lexicon = None
_zipf_cdf = None


def lexicon() -> list[str]:
    global _lexicon, _zipf_cdf
    if _lexicon is None:
        rng = np.random.Generator(np.random.PCG64(LEXICON_SEED))
        words, seen = [], set()
        letters = np.array(list("abcdefghijklmnopqrstuvwxyz"))
        while len(words) < LEXICON_SIZE:
            n = int(rng.integers(2, 11))
            w = "".join(letters[rng.integers(0, 26, size=n)])
            if w not in seen:
                seen.add(w)
                words.append(w)
        _lexicon = words
        p = 1.0 / np.arange(1, LEXICON_SIZE + 1, dtype=np.float64) ** ZIPF_S
        _zipf_cdf = np.cumsum(p / p.sum())
    return _lexicon


def document(seed: int, nbytes: int) -> str:
    """One document of exactly ``nbytes`` UTF-8 bytes (ASCII only)."""
    words = lexicon()
    rng = np.random.Generator(np.random.PCG64(seed))
    parts: list[str] = []
    total = 0
    while total < nbytes:
        paras = []
        for _ in range(int(rng.integers(3, 8))):
            n = int(rng.integers(8, 26))
            idx = np.searchsorted(_zipf_cdf, rng.random(n), side="right")
            idx = np.minimum(idx, LEXICON_SIZE - 1)
            ws = [words[i] for i in idx]
            ws[0] = ws[0].capitalize()
            paras.append(" ".join(ws) + ".")
        p = " ".join(paras)
        parts.append(p)
        total += len(p) + 2
    return "\n\n".join(parts)[:nbytes]


def documents(seeds, nbytes: int) -> list[str]:
    return [document(int(s), nbytes) for s in seeds]


# ---------------------------------------------------------------------------
# random-init arch-2 model
# ---------------------------------------------------------------------------
def rope_tables(ctx: int, theta: float = 10000.0) -> tuple[np.ndarray, np.ndarray]:
    """lut.rs:97-136: angle = pos / theta^(2i/64), Q1.15 with ties-to-even, clamped."""
    cos = np.zeros((ctx, 32), dtype=np.int16)
    sin = np.zeros((ctx, 32), dtype=np.int16)

    def rte(x: float) -> int:   # primitives.rs:253-268 (round_ties_to_even_host)
        fl = math.floor(x)
        diff = x - fl
        if abs(diff - 0.5) < 2.220446049250313e-16:
            return int(fl) if int(fl) % 2 == 0 else int(math.ceil(x))
        return int(fl) + 1 if diff > 0.5 else int(fl)

    for i in range(32):
        freq = 1.0 / math.pow(theta, (2 * i) / 64.0)
        for pos in range(ctx):
            a = pos * freq
            cos[pos, i] = max(-32768, min(32767, rte(math.cos(a) * 32768.0)))
            sin[pos, i] = max(-32768, min(32767, rte(math.sin(a) * 32768.0)))
    return cos, sin


ARCH2 = dict(vocab_size=1024, n_layers=8, n_heads=8, n_kv_heads=2, d_model=512, d_ff=2048,
             head_dim=64)


def arch2_model(shipped: czm.ModelFile, ctx: int, seed: int = 7, arch: dict | None = None) -> bytes:
    """Config-2/4 model bytes: int8 tensors = clamp(round(N(0, 24^2)), +-127) drawn from
    ``seed`` in the fixed order written below; mult/shift, exp LUT, softmax constants
    and tokenizer copied from the shipped model; score_mult = the shipped six values
    followed by its first two.  ``arch`` (keys as ARCH2) builds another shape the same
    way, for tests."""
    a = ARCH2 if arch is None else arch
    d, dff, V, L = a["d_model"], a["d_ff"], a["vocab_size"], a["n_layers"]
    kvd = a["n_kv_heads"] * 64
    rng = np.random.Generator(np.random.PCG64(seed))
    st = shipped.tensors

    def w(*shape):
        x = np.rint(rng.normal(0.0, 24.0, size=shape))
        return np.clip(x, -127, 127).astype(np.int8)

    def sc(name, dtype):
        return np.array(st[name].reshape(()), dtype=dtype)

    sm = st["layers.0.attn.score_mult"].astype(np.int32)
    score_mult = np.concatenate([sm, sm[:2]])[: a["n_heads"]].astype(np.int32)
    t = {"embed.weight": w(V, d)}
    for i in range(L):
        p = f"layers.{i}."
        t[p + "attn_norm.weight"] = w(d)
        t[p + "attn.qkv.weight"] = w(d + 2 * kvd, d)
        t[p + "attn.qkv.mult"] = sc("layers.0.attn.qkv.mult", np.int32)
        t[p + "attn.qkv.shift"] = sc("layers.0.attn.qkv.shift", np.int8)
        t[p + "attn.out.weight"] = w(d, d)
        t[p + "attn.out.mult"] = sc("layers.0.attn.out.mult", np.int32)
        t[p + "attn.out.shift"] = sc("layers.0.attn.out.shift", np.int8)
        t[p + "attn.score_mult"] = score_mult
        t[p + "attn.score_shift"] = sc("layers.0.attn.score_shift", np.int8)
        t[p + "ffn_norm.weight"] = w(d)
        t[p + "post_attn_norm.weight"] = w(d)
        t[p + "ffn.up.weight"] = w(2 * dff, d)
        t[p + "ffn.up.mult"] = sc("layers.0.ffn.up.mult", np.int32)
        t[p + "ffn.up.shift"] = sc("layers.0.ffn.up.shift", np.int8)
        t[p + "ffn.down.weight"] = w(d, dff)
        t[p + "ffn.down.mult"] = sc("layers.0.ffn.down.mult", np.int32)
        t[p + "ffn.down.shift"] = sc("layers.0.ffn.down.shift", np.int8)
        t[p + "post_ffn_norm.weight"] = w(d)
    t["norm.weight"] = w(d)
    t["head.weight"] = w(V, d)
    t["head.mult"] = sc("head.mult", np.int32)
    t["head.shift"] = sc("head.shift", np.int8)
    t["lut.exp2"] = st["lut.exp2"].astype(np.uint16)
    cos, sin = rope_tables(ctx)
    t["lut.rope_cos"] = cos
    t["lut.rope_sin"] = sin
    t["softmax.coef_q24"] = sc("softmax.coef_q24", np.uint32)
    t["softmax.target_total"] = sc("softmax.target_total", np.uint32)
    t["tokenizer.data"] = st["tokenizer.data"].astype(np.uint8)
    meta = dict(shipped.metadata)
    meta.update({k: str(v) for k, v in a.items()})
    meta.update(context_length=str(ctx), context_length_log2=str(int(math.log2(ctx))),
                max_seq_len=str(max(8192, ctx)))
    return czm.write_safetensors(t, meta)
