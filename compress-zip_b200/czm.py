"""The .czm model file: a safetensors container with flat string metadata.

Reader and writer for the layout the reference loads at rust/src/model.rs:108-274
(safetensors parsing at rust/src/safetensors.rs:287-376): an 8-byte little-endian
header length, a JSON header mapping tensor names to dtype / shape /
data_offsets plus a ``__metadata__`` object of strings, then the tensor bytes.
Metadata defaults follow model.rs:113-145.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import numpy as np

_DT = {"I8": np.int8, "I16": np.int16, "I32": np.int32, "I64": np.int64, "U8": np.uint8,
       "U16": np.uint16, "U32": np.uint32, "F16": np.float16, "F32": np.float32,
       "BOOL": np.int32}
_DT_INV = {np.dtype(np.int8): "I8", np.dtype(np.int16): "I16", np.dtype(np.int32): "I32",
           np.dtype(np.int64): "I64", np.dtype(np.uint8): "U8", np.dtype(np.uint16): "U16",
           np.dtype(np.uint32): "U32", np.dtype(np.float16): "F16", np.dtype(np.float32): "F32"}


@dataclass
class ModelConfig:
    """model.rs:19-46 with the loader defaults of model.rs:113-145."""
    vocab_size: int = 1024
    n_layers: int = 1
    n_heads: int = 6
    n_kv_heads: int = 1
    d_model: int = 384
    d_ff: int = 1024
    head_dim: int = 64
    max_seq_len: int = 64
    context_length: int = 64
    rope_theta_q16: int = 655360000


def read_safetensors(data: bytes) -> tuple[dict, dict]:
    if len(data) < 8:
        raise ValueError("Invalid header size")
    (hlen,) = struct.unpack_from("<Q", data, 0)
    if 8 + hlen > len(data):
        raise ValueError("Invalid header size")
    header = json.loads(data[8:8 + hlen].decode("utf-8"))
    if not isinstance(header, dict):
        raise ValueError("Header is not a JSON object")
    meta = {k: v for k, v in (header.pop("__metadata__", None) or {}).items()
            if isinstance(v, str)}
    base = 8 + hlen
    tensors = {}
    for name, info in header.items():
        dt = info["dtype"]
        if dt not in _DT:
            raise ValueError(f"Unknown dtype: {dt}")
        a, b = info["data_offsets"]
        shape = tuple(int(s) for s in info["shape"])
        if base + b > len(data) or a > b:
            raise ValueError(f"tensor {name} out of file bounds")
        arr = np.frombuffer(data, dtype=_DT[dt], count=(b - a) // np.dtype(_DT[dt]).itemsize,
                            offset=base + a)
        tensors[name] = arr.reshape(shape) if shape else arr.reshape(())
    return tensors, meta


def write_safetensors(tensors: dict, metadata: dict) -> bytes:
    header = {"__metadata__": {k: str(v) for k, v in metadata.items()}}
    blobs = []
    off = 0
    for name, arr in tensors.items():
        arr = np.asarray(arr)   # keeps 0-d scalars 0-d (ascontiguousarray would not)
        raw = arr.tobytes()
        header[name] = {"dtype": _DT_INV[arr.dtype], "shape": list(arr.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hj += b" " * ((8 - len(hj) % 8) % 8)
    return struct.pack("<Q", len(hj)) + hj + b"".join(blobs)


class ModelFile:
    """Parsed .czm: config, tensors and the embedded tokenizer bytes."""

    def __init__(self, data: bytes):
        self.raw = data
        self.tensors, self.metadata = read_safetensors(data)
        md = self.metadata

        def pu(key, default):
            try:
                return int(md[key])
            except (KeyError, ValueError):
                return default

        if pu("context_length", -1) >= 0:
            ctx = pu("context_length", 0)
        elif pu("context_length_log2", -1) >= 0:
            ctx = 1 << pu("context_length_log2", 0)
        else:
            ctx = pu("max_seq_len", 64)
        self.config = ModelConfig(
            vocab_size=pu("vocab_size", 1024), n_layers=pu("n_layers", 1),
            n_heads=pu("n_heads", 6), n_kv_heads=pu("n_kv_heads", 1),
            d_model=pu("d_model", 384), d_ff=pu("d_ff", 1024), head_dim=pu("head_dim", 64),
            max_seq_len=pu("max_seq_len", 64), context_length=ctx,
            rope_theta_q16=pu("rope_theta_q16", 655360000))
        self.tokenizer_codec = md.get("tokenizer_codec", "zstd")
        t = self.tensors.get("tokenizer.data")
        self.tokenizer_data = None if t is None else t.tobytes()

    @classmethod
    def load(cls, path: str) -> "ModelFile":
        with open(path, "rb") as f:
            return cls(f.read())

    def tokenizer(self):
        from .tokenizer import Tokenizer

        if self.tokenizer_data is None:
            raise FileNotFoundError("No embedded tokenizer in model")
        return Tokenizer.from_model(self.tokenizer_data, self.tokenizer_codec)
