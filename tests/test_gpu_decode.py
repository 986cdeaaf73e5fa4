"""GPU decompression (czg_decompress_chunks) against the CPU oracle.

Decoding is exact: tokens decoded on the GPU equal the original tokens for
streams produced by the oracle's encoder, equal the oracle decoder's tokens for
arbitrary (corrupt) bytes, and round-trip the GPU's own compressed output.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(shipped_path):
    from compress_zip_b200.engine import Engine

    e = Engine.from_file(shipped_path, 0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def doc_tokens(shipped_path):
    from compress_zip_b200 import czm, synth

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    return [np.array(tok.encode_with_special_tokens(synth.document(s, n)), np.uint32)
            for s, n in ((21, 5000), (22, 2200), (23, 300))]


def _chunked(docs, C):
    toks, starts = [], [0]
    for ids in docs:
        base = sum(len(t) for t in toks)
        for s in range(0, len(ids), C):
            starts.append(base + min(s + C, len(ids)))
        toks.append(ids)
    return np.concatenate(toks), np.array(starts, np.uint64)


@pytest.mark.parametrize("C", [64, 1024])
def test_decode_oracle_streams(eng, shipped_oracle, oracle_mod, doc_tokens, C):
    tokens, starts = _chunked(doc_tokens, C)
    chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
    got = eng.decompress_chunks(chunks, np.diff(starts))
    assert np.array_equal(got, tokens)


def test_decode_into_caller_buffer(eng, shipped_oracle, oracle_mod, doc_tokens):
    """decompress_chunks(out=...): the tokens land in the caller's buffer (reused
    across calls, entries past the result untouched), and a buffer of the wrong
    type or size is refused before any device work."""
    tokens, starts = _chunked(doc_tokens, 256)
    chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
    buf = np.full(len(tokens) + 5, 0xFFFFFFFF, dtype=np.uint32)
    for _ in range(2):
        got = eng.decompress_chunks(chunks, np.diff(starts), out=buf)
        assert np.shares_memory(got, buf) and np.array_equal(got, tokens)
        assert (buf[len(tokens):] == 0xFFFFFFFF).all()
        buf[: len(tokens)] = 0xFFFFFFFF
    with pytest.raises(ValueError):
        eng.decompress_chunks(chunks, np.diff(starts), out=np.empty(len(tokens) - 1, np.uint32))
    with pytest.raises(ValueError):
        eng.decompress_chunks(chunks, np.diff(starts), out=np.empty(len(tokens), np.int64))


def test_gpu_roundtrip_ragged(eng, doc_tokens):
    tokens, starts = _chunked(doc_tokens, 512)
    # an empty chunk and one-token chunks in the middle
    starts = np.concatenate([starts[:2], [starts[1]], [starts[1] + 1], starts[2:]]).astype(np.uint64)
    starts = np.unique(np.concatenate([starts, [starts[1] + 1]])).astype(np.uint64)
    starts = np.sort(np.concatenate([starts, [starts[1]]])).astype(np.uint64)   # repeated = empty chunk
    chunks = eng.compress_chunks(tokens, starts)
    got = eng.decompress_chunks(chunks, np.diff(starts))
    assert np.array_equal(got, tokens)


def test_decode_corrupt_bytes_match_oracle(eng, shipped_oracle, oracle_mod):
    rng = np.random.default_rng(9)
    chunks = [rng.integers(0, 256, int(n), dtype=np.uint8).tobytes() for n in (0, 1, 7, 40, 300)]
    n_tok = np.array([5, 17, 64, 100, 257], np.uint32)
    want = oracle_mod.decompress_chunks(shipped_oracle, chunks, n_tok)
    got = eng.decompress_chunks(chunks, n_tok)
    assert np.array_equal(got, want)


def test_decode_many_streams_small_waves(shipped_path, shipped_oracle, oracle_mod, doc_tokens, monkeypatch):
    """A KV-cache budget that forces several decode waves."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv("CZG_DECODE_KV_BYTES", str(64 * 64 * 128))
    e = Engine.from_file(shipped_path, 0)
    try:
        tokens, starts = _chunked(doc_tokens, 64)
        chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
        assert np.array_equal(e.decompress_chunks(chunks, np.diff(starts)), tokens)
    finally:
        e.close()


def test_decode_arch2(tmp_path, shipped_path, oracle_mod, doc_tokens):
    from compress_zip_b200 import czm, synth
    from compress_zip_b200.engine import Engine

    data = synth.arch2_model(czm.ModelFile.load(shipped_path), 512)
    p = tmp_path / "a2.czm"
    p.write_bytes(data)
    om = oracle_mod.load_model(str(p))
    e = Engine(data, 0)
    try:
        tokens, starts = _chunked([doc_tokens[1]], 512)
        chunks = oracle_mod.compress_chunks(om, tokens, starts)
        assert e.compress_chunks(tokens, starts) == chunks
        assert np.array_equal(e.decompress_chunks(chunks, np.diff(starts)), tokens)
    finally:
        e.close()


def test_decode_many_streams_roundtrip(eng, shipped_path):
    """Thousands of streams of ragged lengths: every GEMM of the lockstep decode
    runs with a shrinking row count over many output tiles per CTA, including
    tiles whose last rows lie beyond the active streams."""
    from compress_zip_b200 import czm, synth

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    docs = tok.encode_batch(synth.documents(range(3000, 3900), 4096), num_threads=8)
    tokens, starts = _chunked([np.asarray(d, np.uint32) for d in docs], 128)
    chunks = eng.compress_chunks(tokens, starts)
    assert len(chunks) > 6000
    got = eng.decompress_chunks(chunks, np.diff(starts))
    assert np.array_equal(got, tokens)


@pytest.mark.parametrize("sink,score_mult", [
    (True, None),
    (False, [1 << 20, 1 << 24, 2147483647, -2147483647, 3, -60000]),   # record-heavy, clamped scores
])
def test_decode_attention_edge_models(tmp_path, shipped_path, oracle_mod, doc_tokens, sink, score_mult):
    """Decode attention with a sink key and with extreme score multipliers (saturated scores)."""
    from compress_zip_b200 import czm
    from compress_zip_b200.engine import Engine

    mf = czm.ModelFile.load(shipped_path)
    t = {k: np.array(v) for k, v in mf.tensors.items()}
    if sink:
        t["layers.0.attn.sink_key"] = np.random.default_rng(11).integers(-127, 128, 64).astype(np.int8)
    if score_mult is not None:
        t["layers.0.attn.score_mult"] = np.asarray(score_mult, np.int32)
    p = tmp_path / "edge.czm"
    p.write_bytes(czm.write_safetensors(t, mf.metadata))
    om = oracle_mod.load_model(str(p))
    e = Engine.from_file(str(p), 0)
    try:
        tokens, starts = _chunked(doc_tokens, 300)
        chunks = oracle_mod.compress_chunks(om, tokens, starts)
        assert np.array_equal(e.decompress_chunks(chunks, np.diff(starts)), tokens)
    finally:
        e.close()


def test_decode_scalar_attention_path(shipped_path, shipped_oracle, oracle_mod, doc_tokens, monkeypatch):
    """The CUDA-core decode attention (used for more than 8 heads) on the shipped model."""
    from compress_zip_b200.engine import Engine

    monkeypatch.setenv("CZG_SCALAR_DECODE", "1")
    e = Engine.from_file(shipped_path, 0)
    try:
        tokens, starts = _chunked(doc_tokens, 256)
        chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
        assert np.array_equal(e.decompress_chunks(chunks, np.diff(starts)), tokens)
    finally:
        e.close()


def test_decode_launch_modes_agree(eng, shipped_oracle, oracle_mod, doc_tokens, monkeypatch):
    """The step kernels under programmatic dependent launch (the default), plain
    launches (CZG_PDL=0) and plain launches with per-kernel events decode the same
    oracle-encoded streams to the original tokens."""
    tokens, starts = _chunked(doc_tokens, 256)
    chunks = oracle_mod.compress_chunks(shipped_oracle, tokens, starts)
    n_tok = np.diff(starts)
    assert np.array_equal(eng.decompress_chunks(chunks, n_tok), tokens)
    monkeypatch.setenv("CZG_PDL", "0")
    assert np.array_equal(eng.decompress_chunks(chunks, n_tok), tokens)
    monkeypatch.delenv("CZG_PDL")
    eng.set_kernel_timing(True)
    try:
        assert np.array_equal(eng.decompress_chunks(chunks, n_tok), tokens)
        assert eng.last_stats()["kernels"]["cdf_decode"]["launches"] > 0
    finally:
        eng.set_kernel_timing(False)
