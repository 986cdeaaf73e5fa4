"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bit-exact on every intermediate exposed by the debug trace (attention output
per layer, final-norm output, int32 logits, coder interval) and on the encoded
chunk bytes.  Inputs: seeded synthetic text through the model's own tokenizer,
plus random token ids for edge cases.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def shipped_engine(shipped_path):
    from compress_zip_b200.engine import Engine

    eng = Engine.from_file(shipped_path, 0)
    yield eng
    eng.close()


@pytest.fixture(scope="module")
def shipped_tokens(shipped_path):
    from compress_zip_b200 import czm, synth

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    return np.array(tok.encode_with_special_tokens(synth.document(0, 15000)), dtype=np.uint32)


def _starts(n, C):
    return np.array(list(range(0, n, C)) + [n], dtype=np.uint64)


def _trace_equal(eng, om, oracle_mod, toks):
    g = eng.debug_trace(toks)
    o = oracle_mod.chunk_trace(om, toks)
    for k in ("attn", "final_in", "logits", "lohi"):
        if not np.array_equal(g[k], o[k]):
            bad = np.argwhere(g[k] != o[k])
            raise AssertionError(f"{k} differs at {len(bad)} places, first {bad[:5].tolist()}")


@pytest.mark.parametrize("n", [1, 2, 33, 64, 300])
def test_trace_shipped(shipped_engine, shipped_oracle, oracle_mod, shipped_tokens, n):
    _trace_equal(shipped_engine, shipped_oracle, oracle_mod, shipped_tokens[:n])


def test_trace_shipped_full_context(shipped_engine, shipped_oracle, oracle_mod, shipped_tokens):
    _trace_equal(shipped_engine, shipped_oracle, oracle_mod, shipped_tokens[1000:2024])


def test_trace_random_tokens(shipped_engine, shipped_oracle, oracle_mod):
    rng = np.random.default_rng(5)
    toks = rng.integers(0, 1024, 200).astype(np.uint32)
    _trace_equal(shipped_engine, shipped_oracle, oracle_mod, toks)


def test_head_cdf_fused_matches_unfused(shipped_path, monkeypatch):
    """The fused head + coder-interval kernel against the head GEMM + CDF pair on the
    same engine build: random token ids (unusual logit rows), ragged chunks and more
    128-row blocks than SMs (several blocks per CTA, the per-quadrant mbarriers
    cycling through their phases)."""
    from compress_zip_b200.engine import Engine

    rng = np.random.default_rng(17)
    lens = rng.integers(1, 1025, 80)   # ~41 K rows: ~320 blocks of 128 over 148 SMs
    starts = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
    toks = rng.integers(0, 1024, int(starts[-1])).astype(np.uint32)
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("CZG_HEAD_CDF", mode)
        e = Engine.from_file(shipped_path, 0)
        try:
            e.set_kernel_timing(True)
            out[mode] = e.compress_chunks(toks, starts)
            stats = e.last_stats()["kernels"]
            assert (stats["head_cdf"]["launches"] > 0) == (mode == "1")
        finally:
            e.close()
    assert out["0"] == out["1"]


@pytest.mark.parametrize("C", [64, 1024])
def test_compress_bytes_match_oracle(shipped_engine, shipped_oracle, oracle_mod, shipped_tokens, C):
    starts = _starts(len(shipped_tokens), C)
    got = shipped_engine.compress_chunks(shipped_tokens, starts)
    want = oracle_mod.compress_chunks(shipped_oracle, shipped_tokens, starts)
    assert len(got) == len(want)
    for i, (a, b) in enumerate(zip(got, want)):
        assert a == b, f"chunk {i} differs"


def test_compress_many_docs(shipped_engine, shipped_oracle, oracle_mod, shipped_path):
    """Several documents with ragged last chunks in one call."""
    from compress_zip_b200 import czm, synth

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    toks, starts = [], [0]
    for seed in (1, 2, 3):
        ids = tok.encode_with_special_tokens(synth.document(seed, 3000 + 700 * seed))
        base = sum(len(t) for t in toks)
        for s in range(0, len(ids), 256):
            starts.append(base + min(s + 256, len(ids)))
        toks.append(ids)
    tokens = np.concatenate([np.array(t, np.uint32) for t in toks])
    starts = np.array(starts, np.uint64)
    got = shipped_engine.compress_chunks(tokens, starts)
    want = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
    assert got == want


def test_compress_waves_and_workspace_growth(shipped_path, shipped_oracle, oracle_mod, monkeypatch):
    """A call spanning several waves (small wave cap), and a workspace that grows
    from a small call to a larger one on the same context (default cap, which starts
    at 65,536 rows); bytes equal the oracle's."""
    from compress_zip_b200 import czm, synth
    from compress_zip_b200.engine import Engine

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    ids = [tok.encode_with_special_tokens(synth.document(seed, 15000)) for seed in range(21, 28)]

    def packed(docs):
        starts, base = [0], 0
        for d in docs:
            for s in range(0, len(d), 1024):
                starts.append(base + min(s + 1024, len(d)))
            base += len(d)
        return np.concatenate([np.array(d, np.uint32) for d in docs]), np.array(starts, np.uint64)

    small, large = packed(ids[:1]), packed(ids)   # ~11 K and ~80 K tokens
    assert len(large[0]) > 65536
    want_small = oracle_mod.compress_chunks(shipped_oracle, *small)
    want_large = oracle_mod.compress_chunks(shipped_oracle, *large)
    for cap in ("16384", None):
        if cap:
            monkeypatch.setenv("CZG_WAVE_TOKENS", cap)
        else:
            monkeypatch.delenv("CZG_WAVE_TOKENS", raising=False)
        e = Engine.from_file(shipped_path, 0)
        try:
            assert e.compress_chunks(*small) == want_small
            assert e.compress_chunks(*large) == want_large
        finally:
            e.close()


def test_edge_cases(shipped_engine, shipped_oracle, oracle_mod):
    from compress_zip_b200.engine import CzgError

    # no chunks
    packed, lens = shipped_engine.compress_packed(np.zeros(0, np.uint32), np.zeros(1, np.uint64))
    assert len(packed) == 0 and len(lens) == 0
    # one-token chunks and an empty chunk
    toks = np.array([5, 1023, 0, 1022], np.uint32)
    starts = np.array([0, 1, 2, 2, 4], np.uint64)
    assert shipped_engine.compress_chunks(toks, starts) == \
        oracle_mod.compress_chunks(shipped_oracle, toks, starts)
    # token id out of range: the reference would panic, the ABI reports it
    with pytest.raises(CzgError) as ei:
        shipped_engine.compress_chunks(np.array([1, 1024], np.uint32), np.array([0, 2], np.uint64))
    assert ei.value.status == 7
    # chunk longer than the model context
    with pytest.raises(CzgError) as ei:
        shipped_engine.compress_chunks(np.zeros(1025, np.uint32), np.array([0, 1025], np.uint64))
    assert ei.value.status == 8
    # the context still works after errors
    assert shipped_engine.compress_chunks(toks, starts) == \
        oracle_mod.compress_chunks(shipped_oracle, toks, starts)


@pytest.fixture(scope="module")
def arch2(tmp_path_factory, shipped_path):
    from compress_zip_b200 import czm, synth
    from compress_zip_b200.engine import Engine

    data = synth.arch2_model(czm.ModelFile.load(shipped_path), 512)
    p = tmp_path_factory.mktemp("m") / "arch2_512.czm"
    p.write_bytes(data)
    eng = Engine(data, 0)
    yield eng, str(p)
    eng.close()


def test_arch2_trace_and_bytes(arch2, oracle_mod, shipped_tokens):
    eng, path = arch2
    om = oracle_mod.load_model(path)
    assert om.check() == 0
    _trace_equal(eng, om, oracle_mod, shipped_tokens[:200])
    toks = shipped_tokens[:1500]
    starts = _starts(len(toks), 512)
    assert eng.compress_chunks(toks, starts) == oracle_mod.compress_chunks(om, toks, starts)


@pytest.mark.parametrize("queue", ["0", "1"])
def test_four_head_model(shipped_path, tmp_path, oracle_mod, shipped_tokens, monkeypatch, queue):
    """A synthetic 4-head model (d 256, 1 KV head, d_ff 512, 2 layers, ctx 1024): the
    d = 256 forms of the QKV K/V epilogue (128-column tiles), the fused norm GEMMs
    and the streamed attention in both schedules; trace and bytes against the oracle,
    and the GPU decodes the oracle's streams."""
    from compress_zip_b200 import czm, synth
    from compress_zip_b200.engine import Engine

    arch = dict(vocab_size=1024, n_layers=2, n_heads=4, n_kv_heads=1, d_model=256, d_ff=512, head_dim=64)
    data = synth.arch2_model(czm.ModelFile.load(shipped_path), 1024, seed=11, arch=arch)
    p = tmp_path / "four_head.czm"
    p.write_bytes(data)
    om = oracle_mod.load_model(str(p))
    assert om.check() == 0
    monkeypatch.setenv("CZG_ATTN_QUEUE", queue)
    eng = Engine(data, 0)
    try:
        _trace_equal(eng, om, oracle_mod, shipped_tokens[:300])
        toks = shipped_tokens[:2500]
        starts = _starts(len(toks), 1024)
        chunks = oracle_mod.compress_chunks(om, toks, starts)
        assert eng.compress_chunks(toks, starts) == chunks
        assert np.array_equal(eng.decompress_chunks(chunks, np.diff(starts)), toks)
    finally:
        eng.close()


def _variant_model(shipped_path, tmp_path, sink=False, score_mult=None):
    """The shipped model with an attention sink key and/or other score multipliers."""
    from compress_zip_b200 import czm

    mf = czm.ModelFile.load(shipped_path)
    t = {k: np.array(v) for k, v in mf.tensors.items()}
    rng = np.random.default_rng(11)
    if sink:
        t["layers.0.attn.sink_key"] = rng.integers(-127, 128, 64).astype(np.int8)
    if score_mult is not None:
        t["layers.0.attn.score_mult"] = np.asarray(score_mult, np.int32)
    data = czm.write_safetensors(t, mf.metadata)
    p = tmp_path / "variant.czm"
    p.write_bytes(data)
    return data, str(p)


@pytest.mark.parametrize("staged", [False, True])
@pytest.mark.parametrize("sink,score_mult", [
    (True, None),
    (False, [1 << 20, 1 << 24, 2147483647, -2147483647, 3, -60000]),   # record-heavy, clamped scores
    (True, [400000, 1, 70000, 58218, -58218, 900000]),
])
def test_attention_edge_models(shipped_path, tmp_path, oracle_mod, shipped_tokens, sink, score_mult, staged,
                               monkeypatch):
    """Both tensor-core chunk attention forms: K/V tiles streamed per warp (the
    default) and the chunk's K/V^T staged in shared memory (CZG_ATTN_STAGED=1)."""
    from compress_zip_b200.engine import Engine

    if staged:
        monkeypatch.setenv("CZG_ATTN_STAGED", "1")
    data, path = _variant_model(shipped_path, tmp_path, sink, score_mult)
    om = oracle_mod.load_model(path)
    eng = Engine(data, 0)
    try:
        _trace_equal(eng, om, oracle_mod, shipped_tokens[:700])
        toks = shipped_tokens[:2100]
        starts = _starts(len(toks), 1024)
        assert eng.compress_chunks(toks, starts) == oracle_mod.compress_chunks(om, toks, starts)
    finally:
        eng.close()


@pytest.mark.parametrize("env", ["CZG_SCALAR_ATTENTION", "CZG_ATTN_STAGED"])
def test_other_attention_kernels(shipped_path, shipped_oracle, oracle_mod, shipped_tokens, monkeypatch, env):
    """The CUDA-core attention kernel and the shared-memory-staged tensor-core kernel,
    each selected by its switch, against the oracle."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv(env, "1")
    eng = Engine.from_file(shipped_path, 0)
    try:
        _trace_equal(eng, shipped_oracle, oracle_mod, shipped_tokens[:300])
        starts = _starts(len(shipped_tokens), 1024)
        assert eng.compress_chunks(shipped_tokens, starts) == \
            oracle_mod.compress_chunks(shipped_oracle, shipped_tokens, starts)
    finally:
        eng.close()


@pytest.mark.parametrize("queue", ["0", "1"])
def test_streamed_attention_schedules(shipped_path, shipped_oracle, oracle_mod, shipped_tokens, monkeypatch, queue):
    """The streamed chunk attention with one CTA per chunk (CZG_ATTN_QUEUE=0) and as a
    persistent grid over a global task queue (CZG_ATTN_QUEUE=1; the default from
    1024-key chunks on), on full and ragged chunks, against the oracle."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv("CZG_ATTN_QUEUE", queue)
    eng = Engine.from_file(shipped_path, 0)
    try:
        for C in (1024, 300):
            starts = _starts(len(shipped_tokens), C)
            assert eng.compress_chunks(shipped_tokens, starts) == \
                oracle_mod.compress_chunks(shipped_oracle, shipped_tokens, starts)
    finally:
        eng.close()


def test_kv_prep_kernel_path(shipped_path, shipped_oracle, oracle_mod, shipped_tokens, monkeypatch):
    """The key rotation and the per-chunk K/V layout from k_kv_prep_split after a plain
    requantising QKV GEMM (CZG_KV_EPILOGUE=0), in place of the QKV epilogue that writes
    them (the default, which every other test runs), against the oracle."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv("CZG_KV_EPILOGUE", "0")
    eng = Engine.from_file(shipped_path, 0)
    try:
        _trace_equal(eng, shipped_oracle, oracle_mod, shipped_tokens[:300])
        starts = _starts(len(shipped_tokens), 1024)
        assert eng.compress_chunks(shipped_tokens, starts) == \
            oracle_mod.compress_chunks(shipped_oracle, shipped_tokens, starts)
    finally:
        eng.close()


@pytest.mark.parametrize("mode", ["ties", "flat", "extreme"])
def test_cdf_edge_models(shipped_path, tmp_path, oracle_mod, shipped_tokens, mode):
    """CDF corner cases through real logits: tied maxima (first index wins),
    a flat row (every weight 65535), and logits far apart (most weights 1); the
    GPU decoder (its own max and first-argmax search) decodes the oracle's bytes
    back to the tokens."""
    from compress_zip_b200 import czm
    from compress_zip_b200.engine import Engine

    mf = czm.ModelFile.load(shipped_path)
    t = {k: np.array(v) for k, v in mf.tensors.items()}
    hw = t["head.weight"].copy()
    if mode == "ties":
        hw[1::2] = hw[0::2]                       # logits of tokens 2k and 2k+1 are equal
    elif mode == "flat":
        hw[:] = 0                                 # every logit is 0
    else:
        hw = np.where(hw >= 0, 127, -127).astype(np.int8)
    t["head.weight"] = hw
    p = tmp_path / f"cdf_{mode}.czm"
    p.write_bytes(czm.write_safetensors(t, mf.metadata))
    om = oracle_mod.load_model(str(p))
    eng = Engine.from_file(str(p), 0)
    try:
        _trace_equal(eng, om, oracle_mod, shipped_tokens[:400])
        toks = shipped_tokens[:1500]
        starts = _starts(len(toks), 512)
        want = oracle_mod.compress_chunks(om, toks, starts)
        assert eng.compress_chunks(toks, starts) == want
        assert np.array_equal(eng.decompress_chunks(want, np.diff(starts).astype(np.uint32)), toks)
    finally:
        eng.close()


@pytest.mark.parametrize("env", ["CZG_RESIDUAL32", "CZG_INT_REQUANT"])
def test_int32_residual_path(shipped_path, shipped_oracle, oracle_mod, shipped_tokens, monkeypatch, env):
    """The int32 residual stream (used for models deeper than 128 layers), and the
    32-bit integer requantisation epilogue in place of the FP32 one, on the shipped model."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv(env, "1")
    eng = Engine.from_file(shipped_path, 0)
    try:
        _trace_equal(eng, shipped_oracle, oracle_mod, shipped_tokens[:300])
        starts = _starts(len(shipped_tokens), 1024)
        assert eng.compress_chunks(shipped_tokens, starts) == \
            oracle_mod.compress_chunks(shipped_oracle, shipped_tokens, starts)
    finally:
        eng.close()


def test_config4_long_chunks(tmp_path, shipped_path, oracle_mod, monkeypatch):
    """Configuration-4 shape: the arch-2 model at context 4096 with chunks longer
    than 1024 positions next to short ones (the tensor-core attention streaming
    K/V tiles from the per-chunk layout), compressed bytes equal to the oracle's
    and to the CUDA-core attention's, and decoded back on the GPU."""
    from compress_zip_b200 import czm, synth
    from compress_zip_b200.engine import Engine

    mf = czm.ModelFile.load(shipped_path)
    data = synth.arch2_model(mf, 4096)
    p = tmp_path / "arch2_4096.czm"
    p.write_bytes(data)
    om = oracle_mod.load_model(str(p))
    toks = np.array(mf.tokenizer().encode_with_special_tokens(synth.document(10000, 4000)), np.uint32)[:2500]
    starts = np.array([0, 1300, 1337, 2500], np.uint64)
    eng = Engine(data, 0)
    try:
        want = oracle_mod.compress_chunks(om, toks, starts)
        got = eng.compress_chunks(toks, starts)
        assert got == want
        assert np.array_equal(eng.decompress_chunks(got, np.diff(starts).astype(np.uint32)), toks)
    finally:
        eng.close()
    monkeypatch.setenv("CZG_SCALAR_ATTENTION", "1")
    eng = Engine(data, 0)
    try:
        assert eng.compress_chunks(toks, starts) == want
    finally:
        eng.close()


@pytest.mark.parametrize("proj,mult,shift", [
    ("ffn.up", 819, 10),          # |mult| >= 2^(shift-1): clamped 32-bit requantisation
    ("ffn.down", 1 << 28, 30),    # product beyond 32 bits: 64-bit requantisation
    ("attn.qkv", -3000, 16),      # negative multiplier (FP32 form)
    ("ffn.up", 1, 2),             # tiny multiplier: FP32 form, clamp bound 509
    ("attn.out", (1 << 22) + 1, 24),   # M1 - M1 * mult / 2^shift not an exact float: 32-bit clamped form
    ("attn.out", (1 << 23) + 1, 30),   # clamp bound * mult beyond 32 bits: 64-bit form
])
def test_requant_forms(shipped_path, tmp_path, oracle_mod, shipped_tokens, proj, mult, shift):
    """Each requantisation form of the GEMM epilogue against the oracle."""
    from compress_zip_b200 import czm
    from compress_zip_b200.engine import Engine

    mf = czm.ModelFile.load(shipped_path)
    t = {k: np.array(v) for k, v in mf.tensors.items()}
    t[f"layers.0.{proj}.mult"] = np.asarray(mult, np.int32)
    t[f"layers.0.{proj}.shift"] = np.asarray(shift, np.int8)
    p = tmp_path / "rq.czm"
    p.write_bytes(czm.write_safetensors(t, mf.metadata))
    om = oracle_mod.load_model(str(p))
    eng = Engine.from_file(str(p), 0)
    try:
        _trace_equal(eng, om, oracle_mod, shipped_tokens[:300])
        toks = shipped_tokens[:1100]
        starts = _starts(len(toks), 512)
        assert eng.compress_chunks(toks, starts) == oracle_mod.compress_chunks(om, toks, starts)
    finally:
        eng.close()


def test_dff_not_multiple_of_128(shipped_path, tmp_path, oracle_mod, shipped_tokens):
    """d_ff = 960 (a multiple of 64, not of 128): the engine pads the FFN to 1024 hidden
    units with zero weights for its tcgen05 GEMMs; bytes and intermediates equal the
    oracle's, which runs the unpadded 960."""
    from compress_zip_b200 import czm
    from compress_zip_b200.engine import Engine

    mf = czm.ModelFile.load(shipped_path)
    t = {k: np.array(v) for k, v in mf.tensors.items()}
    dff, new = 1024, 960
    up = t["layers.0.ffn.up.weight"].reshape(2 * dff, -1)
    t["layers.0.ffn.up.weight"] = np.ascontiguousarray(np.concatenate([up[:new], up[dff:dff + new]]))
    t["layers.0.ffn.down.weight"] = np.ascontiguousarray(t["layers.0.ffn.down.weight"].reshape(-1, dff)[:, :new])
    meta = dict(mf.metadata)
    meta["d_ff"] = str(new)
    p = tmp_path / "dff960.czm"
    p.write_bytes(czm.write_safetensors(t, meta))
    om = oracle_mod.load_model(str(p))
    assert om.cfg["d_ff"] == new
    eng = Engine.from_file(str(p), 0)
    try:
        assert eng.info["d_ff"] == new
        _trace_equal(eng, om, oracle_mod, shipped_tokens[:300])
        toks = shipped_tokens[:2100]
        starts = _starts(len(toks), 1024)
        got = eng.compress_chunks(toks, starts)
        assert got == oracle_mod.compress_chunks(om, toks, starts)
        assert np.array_equal(eng.decompress_chunks(got, np.diff(starts).astype(np.uint32)), toks)
    finally:
        eng.close()


def test_capacity_and_pipelined_waves(shipped_path, shipped_oracle, oracle_mod, shipped_tokens, monkeypatch):
    """Several pipelined waves (small wave cap): an output buffer one byte short gives
    CZG_E_CAPACITY with the exact size, the context stays usable, and with room the
    packed bytes and lengths equal the oracle's; from host and from device tokens."""
    import ctypes as C

    import torch

    from compress_zip_b200 import engine as E

    monkeypatch.setenv("CZG_WAVE_TOKENS", "16384")
    toks = np.concatenate([shipped_tokens] * 6)[:60000].astype(np.uint32)
    starts = _starts(len(toks), 1024)
    want = oracle_mod.compress_chunks(shipped_oracle, toks, starts)
    need_total = sum(len(w) for w in want)
    eng = E.Engine.from_file(shipped_path, 0)
    try:
        L = E.lib()
        n = len(starts) - 1
        lens = np.zeros(n, np.uint32)
        need = C.c_uint64(0)
        out = np.zeros(need_total - 1, np.uint8)
        st = L.czg_compress_chunks(eng._h, toks.ctypes.data, starts.ctypes.data, n, out.ctypes.data, len(out),
                                   lens.ctypes.data, C.byref(need))
        assert st == 4   # CZG_E_CAPACITY
        assert need.value == need_total
        out = np.zeros(need_total, np.uint8)
        st = L.czg_compress_chunks(eng._h, toks.ctypes.data, starts.ctypes.data, n, out.ctypes.data, len(out),
                                   lens.ctypes.data, C.byref(need))
        assert st == 0 and need.value == need_total
        assert out.tobytes() == b"".join(want) and list(lens) == [len(w) for w in want]
        d_tok = torch.from_numpy(toks.view(np.int32)).cuda()
        out2 = np.zeros(need_total, np.uint8)
        assert eng.compress_device(d_tok.data_ptr(), starts, out2, lens) == need_total
        assert out2.tobytes() == b"".join(want)
    finally:
        eng.close()
