"""compress / decompress with the reference CLI's flags (rust/src/main.rs:18-74).

    python compress-zip_b200/cli.py compress   -m MODEL.czm -i in.txt  -o out.czip [-t tok.json] [-c brotli|zstd] [-L 1..5]
    python compress-zip_b200/cli.py decompress -m MODEL.czm -i in.czip -o out.txt  [-t tok.json]

The host steps follow rust/src/main.rs: model and tokenizer loading (124-175),
chunk size from the level (113-122, 186-201), model_id_hash = the first 8 hex
digits of md5 of the model path as given (79-85), the CZIPv1 container and the
outer codec (241-281, 339-365).  The per-chunk model + coder loops
(206-238, 377-396) run on the GPU through the C ABI (engine.py).
"""
from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys
import time

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from __graft_entry__ import load_package

    load_package()
    from compress_zip_b200 import container, czm, outer_codec  # noqa: E402
    from compress_zip_b200.engine import Engine  # noqa: E402
    from compress_zip_b200.tokenizer import Tokenizer  # noqa: E402
else:
    from . import container, czm, outer_codec
    from .engine import Engine
    from .tokenizer import Tokenizer

import numpy as np


def hash_model_path(path: str) -> int:
    """main.rs:79-85: int(md5(path string).hexdigest()[:8], 16)."""
    return int(hashlib.md5(path.encode("utf-8", "surrogateescape")).hexdigest()[:8], 16)


def level_to_context_length(level: int) -> int:
    return {1: 64, 2: 128, 3: 256, 4: 512, 5: 1024}.get(level, 64)   # main.rs:113-122


def _tokenizer(mf: czm.ModelFile, tokenizer_path: str | None) -> Tokenizer:
    if tokenizer_path:
        print(f"Loading tokenizer from {tokenizer_path!r}...")
        with open(tokenizer_path, "rb") as f:
            return Tokenizer.from_json_bytes(f.read())
    print("Loading embedded tokenizer from model...")
    return mf.tokenizer()


def compress(model_path: str, tokenizer_path: str | None, input_path: str, output_path: str,
             codec_str: str = "brotli", level: int | None = None, device: int = 0) -> dict:
    t_total = time.perf_counter()
    codec = {"zstd": container.ZSTD, "brotli": container.BROTLI}.get(codec_str.lower())
    if codec is None:
        raise ValueError(f"Unknown codec: {codec_str}")
    print(f"Loading model from {model_path!r}...")
    mf = czm.ModelFile.load(model_path)
    tok = _tokenizer(mf, tokenizer_path)
    print(f"Reading input from {input_path!r}...")
    with open(input_path, "rb") as f:
        raw = f.read()
    text = raw.decode("utf-8")   # fs::read_to_string: UTF-8 required
    input_bytes = len(raw)
    print("Tokenizing...")
    tokens = np.asarray(tok.encode_with_special_tokens(text), dtype=np.uint32)
    n = len(tokens)
    print(f"  {input_bytes} bytes -> {n} tokens")
    print("Compressing...")
    t_enc = time.perf_counter()
    ctx_len = mf.config.context_length
    if level is not None:
        requested = level_to_context_length(level)
        if requested > ctx_len:   # main.rs:186-197
            print(f"Warning: Level {level} requires {requested} tokens but model only supports "
                  f"{ctx_len}. Using model's context length.", file=sys.stderr)
            chunk_size = ctx_len
        else:
            chunk_size = requested
    else:
        chunk_size = ctx_len
    log2 = int(math.log2(chunk_size)) & 0xFF
    n_chunks = (n + chunk_size - 1) // chunk_size
    starts = np.array([min(i * chunk_size, n) for i in range(n_chunks + 1)], dtype=np.uint64)
    eng = Engine(mf.raw, device)
    try:
        chunks = eng.compress_chunks(tokens, starts) if n_chunks else []
    finally:
        eng.close()
    cf = container.CompressedFile.with_context_length(hash_model_path(model_path), 0, codec,
                                                      input_bytes & 0xFFFFFFFF, log2)
    for i, data in enumerate(chunks):
        is_last = i == n_chunks - 1
        last = int(starts[i + 1] - starts[i]) if is_last else chunk_size
        cf.add_chunk(data, is_last, last & 0xFFFF)
    t_enc = time.perf_counter() - t_enc
    print(f"Writing output to {output_path!r}...")
    outer, payload = cf.to_bytes_uncompressed()
    body = outer_codec.compress(payload, codec)
    with open(output_path, "wb") as f:
        f.write(outer)
        f.write(body)
    out_bytes = len(outer) + len(body)
    total = time.perf_counter() - t_total
    print("\n=== Compression Results ===")
    print(f"Input:  {input_bytes} bytes ({n} tokens)")
    print(f"Output: {out_bytes} bytes")
    if out_bytes:
        print(f"Ratio:  {input_bytes / out_bytes:.2f}x ({100.0 * out_bytes / max(1, input_bytes):.2f}%)")
    if n:
        print(f"Bits per token: {8.0 * out_bytes / n:.2f}")
    print(f"\nEncode time: {t_enc:.2f}s ({n / max(t_enc, 1e-9):.1f} tokens/sec)")
    print(f"Total time:  {total:.2f}s")
    return {"input_bytes": input_bytes, "tokens": n, "output_bytes": out_bytes, "encode_s": t_enc}


def decompress(model_path: str, tokenizer_path: str | None, input_path: str, output_path: str,
               device: int = 0) -> dict:
    t_total = time.perf_counter()
    print(f"Loading model from {model_path!r}...")
    mf = czm.ModelFile.load(model_path)
    tok = _tokenizer(mf, tokenizer_path)
    print(f"Reading compressed file from {input_path!r}...")
    with open(input_path, "rb") as f:
        blob = f.read()
    outer = container.OuterHeader.from_bytes(blob[:container.OUTER_HEADER_SIZE])
    payload = outer_codec.decompress(blob[container.OUTER_HEADER_SIZE:], outer.codec_id)
    cf = container.CompressedFile.read_from_decompressed(outer, payload)
    n_chunks = cf.inner.chunk_count
    counts = np.array([cf.chunk_tokens(i) for i in range(n_chunks)], dtype=np.uint32)
    print(f"  {n_chunks} chunks, {cf.total_tokens()} tokens total")
    print("Decompressing...")
    t_dec = time.perf_counter()
    eng = Engine(mf.raw, device)
    try:
        tokens = eng.decompress_chunks(cf.chunks, counts) if n_chunks else np.zeros(0, np.uint32)
    finally:
        eng.close()
    t_dec = time.perf_counter() - t_dec
    print("Detokenizing...")
    out = tok.decode_bytes(tokens)
    text = out.decode("utf-8", errors="replace")   # String::from_utf8_lossy
    print(f"Writing output to {output_path!r}...")
    with open(output_path, "wb") as f:
        f.write(text.encode("utf-8"))
    total = time.perf_counter() - t_total
    print("\n=== Decompression Results ===")
    print(f"Tokens: {len(tokens)}")
    print(f"Output: {len(out)} bytes")
    print(f"\nDecode time: {t_dec:.2f}s ({len(tokens) / max(t_dec, 1e-9):.1f} tokens/sec)")
    print(f"Total time:  {total:.2f}s")
    return {"tokens": len(tokens), "decode_s": t_dec}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="compress_zip",
                                 description="Neural text compression using a small transformer model")
    sub = ap.add_subparsers(dest="command", required=True)
    c = sub.add_parser("compress", help="Compress a text file")
    c.add_argument("-m", "--model", required=True)
    c.add_argument("-t", "--tokenizer")
    c.add_argument("-i", "--input", required=True)
    c.add_argument("-o", "--output", required=True)
    c.add_argument("-c", "--codec", default="brotli")
    c.add_argument("-L", "--level", type=int, choices=range(1, 6))
    d = sub.add_parser("decompress", help="Decompress a compressed file")
    d.add_argument("-m", "--model", required=True)
    d.add_argument("-t", "--tokenizer")
    d.add_argument("-i", "--input", required=True)
    d.add_argument("-o", "--output", required=True)
    a = ap.parse_args(argv)
    try:
        if a.command == "compress":
            compress(a.model, a.tokenizer, a.input, a.output, a.codec, a.level)
        else:
            decompress(a.model, a.tokenizer, a.input, a.output)
    except Exception as e:   # main.rs:450-453: print the error, exit 1
        print(f"Error: {e}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
