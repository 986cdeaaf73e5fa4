"""The native command line (compress-zip_b200/czg-cli): its host parts without a
GPU -- MD5 of the model path, the outer codecs called exactly as the Python host
layer calls them (identical bytes), container round trips, usage errors."""
import os
import subprocess

import pytest


@pytest.fixture(scope="module")
def cli_bin(root):
    from compress_zip_b200 import build as B

    path = os.path.join(root, "compress-zip_b200", "czg-cli")
    if not os.path.exists(path):
        B.build()
    return path


def run(cli_bin, *args, check=True):
    r = subprocess.run([cli_bin, *args], capture_output=True, text=True, timeout=120)
    if check:
        assert r.returncode == 0, r.stderr
    return r


def test_selftest(cli_bin):
    assert "selftest ok" in run(cli_bin, "selftest").stdout


@pytest.mark.parametrize("path", ["models/v001_eng.czm", "/abs/path/model.czm", "", "mödel 中.czm"])
def test_model_path_hash(cli_bin, path):
    from compress_zip_b200.cli import hash_model_path

    assert run(cli_bin, "md5-path", path).stdout.strip() == "%08x" % hash_model_path(path)


@pytest.mark.parametrize("codec", ["zstd", "brotli"])
def test_outer_codec_bytes(cli_bin, tmp_path, codec):
    from compress_zip_b200 import outer_codec, synth

    data = synth.document(4, 30000).encode() + bytes(range(256)) * 40
    src = tmp_path / "in.bin"
    src.write_bytes(data)
    packed = tmp_path / "packed"
    run(cli_bin, "outer", codec, "compress", str(src), str(packed))
    ref = outer_codec.zstd_compress(data, 22) if codec == "zstd" else outer_codec.brotli_compress(data, 11, 22)
    assert packed.read_bytes() == ref
    back = tmp_path / "back"
    run(cli_bin, "outer", codec, "decompress", str(packed), str(back))
    assert back.read_bytes() == data
    empty = tmp_path / "empty"
    empty.write_bytes(b"")
    run(cli_bin, "outer", codec, "compress", str(empty), str(packed))
    run(cli_bin, "outer", codec, "decompress", str(packed), str(back))
    assert back.read_bytes() == b""


def test_usage_errors(cli_bin, tmp_path):
    assert run(cli_bin, check=False).returncode == 2
    assert run(cli_bin, "compress", "-m", "x", check=False).returncode == 2
    assert run(cli_bin, "compress", "-m", "x", "-i", "y", "-o", "z", "-L", "9", check=False).returncode == 2
    assert run(cli_bin, "frobnicate", "-m", "x", "-i", "y", "-o", "z", check=False).returncode == 2
    bad = tmp_path / "bad"
    bad.write_bytes(b"\x00" * 10)
    r = run(cli_bin, "outer", "brotli", "decompress", str(bad), str(tmp_path / "o"), check=False)
    assert r.returncode == 1 and "Error" in r.stderr
