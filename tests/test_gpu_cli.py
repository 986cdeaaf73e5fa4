"""The drop-in CLI end to end on the GPU: compress -> .czip -> decompress gives
the input text back, and the .czip's inner payload holds exactly the chunk bytes
the CPU oracle produces (shipped model, L1, brotli,
15,000-byte document from seed 0)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("codec,level", [("brotli", 1), ("zstd", 5), ("brotli", None)])
def test_cli_roundtrip_and_payload(tmp_path, shipped_path, shipped_oracle, oracle_mod, codec, level):
    from compress_zip_b200 import cli, container, czm, outer_codec, synth

    text = synth.document(0, 15000)
    src = tmp_path / "in.txt"
    src.write_bytes(text.encode())
    out = tmp_path / "out.czip"
    back = tmp_path / "back.txt"
    cli.compress(shipped_path, None, str(src), str(out), codec, level)
    cli.decompress(shipped_path, None, str(out), str(back))
    assert back.read_bytes() == text.encode()

    blob = out.read_bytes()
    outer = container.OuterHeader.from_bytes(blob[:16])
    payload = outer_codec.decompress(blob[16:], outer.codec_id)
    cf = container.CompressedFile.read_from_decompressed(outer, payload)
    C = {1: 64, 5: 1024, None: 1024}[level]
    ids = np.array(czm.ModelFile.load(shipped_path).tokenizer().encode_with_special_tokens(text), np.uint32)
    starts = np.array(list(range(0, len(ids), C)) + [len(ids)], np.uint64)
    want = oracle_mod.compress_chunks(shipped_oracle, ids, starts)
    assert cf.chunks == want
    assert cf.inner.context_length_log2 == {64: 6, 1024: 10}[C]
    assert cf.inner.model_id_hash == cli.hash_model_path(shipped_path)
    assert outer.uncompressed_len == len(text.encode())


def test_cli_errors(tmp_path, shipped_path):
    from compress_zip_b200 import cli

    src = tmp_path / "in.txt"
    src.write_bytes(b"hello")
    assert cli.main(["compress", "-m", shipped_path, "-i", str(src), "-o", str(tmp_path / "o"),
                     "-c", "lzma"]) == 1
    bad = tmp_path / "bad.czip"
    bad.write_bytes(b"NOTCZIP" + bytes(20))
    assert cli.main(["decompress", "-m", shipped_path, "-i", str(bad), "-o", str(tmp_path / "x")]) == 1
    empty = tmp_path / "empty.txt"
    empty.write_bytes(b"")
    out = tmp_path / "e.czip"
    assert cli.main(["compress", "-m", shipped_path, "-i", str(empty), "-o", str(out), "-L", "3"]) == 0
    assert cli.main(["decompress", "-m", shipped_path, "-i", str(out), "-o", str(tmp_path / "e.txt")]) == 0
    assert (tmp_path / "e.txt").read_bytes() == b""


@pytest.mark.parametrize("codec,level", [("brotli", None), ("zstd", 1), ("brotli", 4)])
def test_native_cli_matches_python_cli(tmp_path, shipped_path, root, codec, level):
    """czg-cli writes the same .czip bytes as the Python host layer, and each
    decompresses the other's file back to the input text."""
    import os
    import subprocess

    from compress_zip_b200 import cli, synth

    exe = os.path.join(root, "compress-zip_b200", "czg-cli")
    text = synth.document(11, 20000) + "\n<|eos|>tail é中\U0001F600\n"
    src = tmp_path / "in.txt"
    src.write_bytes(text.encode())
    py_out, nat_out = tmp_path / "py.czip", tmp_path / "nat.czip"
    cli.compress(shipped_path, None, str(src), str(py_out), codec, level)
    args = [exe, "compress", "-m", shipped_path, "-i", str(src), "-o", str(nat_out), "-c", codec]
    if level:
        args += ["-L", str(level)]
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert nat_out.read_bytes() == py_out.read_bytes()
    for f in (py_out, nat_out):
        back = tmp_path / (f.name + ".txt")
        r = subprocess.run([exe, "decompress", "-m", shipped_path, "-i", str(f), "-o", str(back)],
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        assert back.read_bytes() == text.encode()


def test_native_cli_errors(tmp_path, shipped_path, root):
    import os
    import subprocess

    exe = os.path.join(root, "compress-zip_b200", "czg-cli")
    bad_text = tmp_path / "bad.txt"
    bad_text.write_bytes(b"ok \xff\xfe not utf-8")
    r = subprocess.run([exe, "compress", "-m", shipped_path, "-i", str(bad_text), "-o", str(tmp_path / "o")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 1 and "UTF-8" in r.stderr   # main.rs:170 reads with read_to_string
    bad = tmp_path / "bad.czip"
    bad.write_bytes(b"NOTCZIP" + bytes(20))
    r = subprocess.run([exe, "decompress", "-m", shipped_path, "-i", str(bad), "-o", str(tmp_path / "x")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 1
    empty = tmp_path / "empty.txt"
    empty.write_bytes(b"")
    out = tmp_path / "e.czip"
    assert subprocess.run([exe, "compress", "-m", shipped_path, "-i", str(empty), "-o", str(out), "-L", "3"],
                          capture_output=True, timeout=600).returncode == 0
    assert subprocess.run([exe, "decompress", "-m", shipped_path, "-i", str(out), "-o", str(tmp_path / "e.txt")],
                          capture_output=True, timeout=600).returncode == 0
    assert (tmp_path / "e.txt").read_bytes() == b""
