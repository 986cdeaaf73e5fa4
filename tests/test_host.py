"""Host-side layers (CPU): CZIPv1 container (tests of rust/src/file_format.rs:422-535
restated), outer codecs, the .czm reader, tokenizer, model-path hash."""
import hashlib

import numpy as np
import pytest


def test_outer_header_roundtrip():
    from compress_zip_b200 import container as K

    h = K.OuterHeader(K.ZSTD, 1000, 20)
    h.set_multifile(True)
    b = h.to_bytes()
    assert len(b) == K.OUTER_HEADER_SIZE
    p = K.OuterHeader.from_bytes(b)
    assert (p.codec_id, p.uncompressed_len, p.header_len, p.is_multifile()) == (K.ZSTD, 1000, 20, True)
    with pytest.raises(K.FormatError):
        K.OuterHeader.from_bytes(b"CZIPv2" + b[6:])
    with pytest.raises(K.FormatError):
        K.OuterHeader.from_bytes(b[:7] + bytes([7]) + b[8:])
    with pytest.raises(K.FormatError):
        K.OuterHeader.from_bytes(b[:10])


def test_inner_header_roundtrip():
    from compress_zip_b200 import container as K

    h = K.InnerHeader(0x12345678, 0, 6, 32, [100, 150, 80])
    b = h.to_bytes()
    assert len(b) == h.header_size()
    p = K.InnerHeader.from_bytes(b)
    assert (p.model_id_hash, p.chunk_count, p.last_chunk_tokens, p.chunk_byte_lens) == \
        (0x12345678, 3, 32, [100, 150, 80])
    assert K.InnerHeader.from_bytes(b[:11] + b"\x00" + b[12:]).context_length_log2 == 6  # 0 -> default


def test_file_roundtrip_and_tokens():
    from compress_zip_b200 import container as K

    cf = K.CompressedFile.with_context_length(0x12345678, 1, K.BROTLI, 2000, 6)
    cf.add_chunk(bytes([1, 2, 3, 4, 5]), False, 64)
    cf.add_chunk(bytes([6, 7, 8]), False, 64)
    cf.add_chunk(bytes([9, 10]), True, 48)
    outer, payload = cf.to_bytes_uncompressed()
    p = K.CompressedFile.read_from_decompressed(K.OuterHeader.from_bytes(outer), payload)
    assert p.outer.codec_id == K.BROTLI and p.outer.uncompressed_len == 2000
    assert p.inner.tokenizer_id == 1 and p.inner.chunk_count == 3 and p.inner.last_chunk_tokens == 48
    assert p.chunks == [bytes([1, 2, 3, 4, 5]), bytes([6, 7, 8]), bytes([9, 10])]
    assert p.total_tokens() == 64 + 64 + 48
    assert [p.chunk_tokens(i) for i in range(3)] == [64, 64, 48]
    with pytest.raises(K.FormatError):
        K.CompressedFile.read_from_decompressed(p.outer, payload[:-1])
    cf2 = K.CompressedFile.with_context_length(1, 0, K.ZSTD, 0, 7)
    cf2.add_chunk(b"ab", False, 128)
    cf2.add_chunk(b"c", True, 100)
    o2, p2 = cf2.to_bytes_uncompressed()
    q = K.CompressedFile.read_from_decompressed(K.OuterHeader.from_bytes(o2), p2)
    assert q.inner.tokens_per_chunk() == 128 and q.total_tokens() == 228
    empty = K.CompressedFile.with_context_length(1, 0, K.ZSTD, 0, 10)
    assert empty.total_tokens() == 0 and empty.inner.last_chunk_tokens == 1024
    with pytest.raises(K.FormatError):
        empty.add_chunk(bytes(65536), True, 1)


@pytest.mark.parametrize("codec", [0, 1])
def test_outer_codec_roundtrip(codec):
    from compress_zip_b200 import outer_codec

    rng = np.random.default_rng(codec)
    for n in (0, 1, 1000, 300000):
        data = bytes(rng.integers(0, 8, n, dtype=np.uint8))
        assert outer_codec.decompress(outer_codec.compress(data, codec), codec) == data
    with pytest.raises(ValueError):
        outer_codec.compress(b"x", 5)


def test_zstd_frame_has_no_content_size():
    """zstd::encode_all streams without a pledged size: no content-size field."""
    from compress_zip_b200 import outer_codec

    z = outer_codec.zstd_compress(b"hello world" * 100, 22)
    assert z[:4] == b"\x28\xb5\x2f\xfd"
    fhd = z[4]
    assert (fhd >> 6) == 0 and not (fhd & 0x20)   # FCS flag 0 and not single-segment


def test_czm_reader_matches_safetensors(shipped_path):
    from safetensors import safe_open

    from compress_zip_b200 import czm

    mf = czm.ModelFile.load(shipped_path)
    with safe_open(shipped_path, "np") as f:
        assert mf.metadata == f.metadata()
        for k in f.keys():
            assert np.array_equal(mf.tensors[k], f.get_tensor(k)), k
    assert mf.config.context_length == 1024 and mf.config.max_seq_len == 8192
    blob = czm.write_safetensors(mf.tensors, mf.metadata)
    again = czm.ModelFile(blob)
    for k, v in mf.tensors.items():
        assert np.array_equal(again.tensors[k], v)


def test_tokenizer_roundtrip(shipped_path):
    from compress_zip_b200 import czm, synth

    tok = czm.ModelFile.load(shipped_path).tokenizer()
    text = synth.document(5, 3000) + "<|bos|>Tail<|eos|>"
    ids = tok.encode_with_special_tokens(text)
    assert 1022 in ids and 1023 in ids and max(ids) < 1024
    assert tok.decode_bytes(ids).decode() == text
    with pytest.raises(ValueError):
        tok.decode_bytes([5000])


def test_model_path_hash():
    from compress_zip_b200.cli import hash_model_path

    p = "models/v001_eng.czm"
    assert hash_model_path(p) == int(hashlib.md5(p.encode()).hexdigest()[:8], 16)


def test_arch2_model_shape(shipped_path, oracle_mod):
    from compress_zip_b200 import czm, synth

    data = synth.arch2_model(czm.ModelFile.load(shipped_path), 512)
    mf = czm.ModelFile(data)
    c = mf.config
    assert (c.d_model, c.n_layers, c.n_heads, c.n_kv_heads, c.d_ff, c.context_length) == (512, 8, 8, 2, 2048, 512)
    assert mf.tensors["layers.0.attn.qkv.weight"].shape == (768, 512)
    assert mf.tensors["lut.rope_cos"].shape == (512, 32)
    om = oracle_mod.OracleModel(mf.tensors, mf.metadata)
    assert om.check() == 0
