"""BPE tokenizer of a .czm model (host pre/post step, outside the GPU path).

The reference embeds a zstd- or brotli-compressed tiktoken JSON in the model
(``tokenizer.data``, decoded at rust/src/main.rs:88-109 and 157-163) and
encodes with special tokens allowed (rust/src/tiktoken.rs:498-501).  JSON keys
map one codepoint to one byte (tiktoken.rs:517-527).

The native tokenizer (``libczg_tok.so``, ``csrc/bpe_tokenizer.cpp``, C ABI in
``include/czg_tok.h``) runs it for the pre-tokenizer pattern of the shipped
tokenizers, with a threaded batch encoder; a JSON with any other pattern runs
through the ``tiktoken`` package, the same regex-and-merge algorithm.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np

from . import outer_codec

_HERE = os.path.dirname(os.path.abspath(__file__))
_TOK_LIB = os.path.join(_HERE, "libczg_tok.so")
_lib = None


def native_lib():
    """The native tokenizer library, built on first use (host C++, no GPU needed)."""
    global _lib
    if _lib is None:
        if not os.path.exists(_TOK_LIB):
            from . import build as B

            B.build_tokenizer()
        L = C.CDLL(_TOK_LIB)
        L.czg_tok_create.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(C.c_void_p)]
        L.czg_tok_destroy.argtypes = [C.c_void_p]
        L.czg_tok_last_error.argtypes = [C.c_void_p]
        L.czg_tok_last_error.restype = C.c_char_p
        L.czg_tok_pattern.restype = C.c_char_p
        L.czg_tok_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                     C.POINTER(C.c_size_t)]
        L.czg_tok_encode_batch.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_int]
        L.czg_tok_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                     C.POINTER(C.c_size_t)]
        _lib = L
    return _lib


E_PATTERN = 3


def _utf8(text: str) -> bytes:
    try:
        return text.encode("utf-8")
    except UnicodeEncodeError:   # lone surrogates: replaced, as tiktoken does
        return text.encode("utf-16", "surrogatepass").decode("utf-16", "replace").encode("utf-8")


class NativeTokenizer:
    """czg_tok handle: encode / encode_batch / decode_bytes of the reference's CoreBPE."""

    def __init__(self, json_bytes: bytes):
        L = native_lib()
        h = C.c_void_p()
        st = L.czg_tok_create(json_bytes, len(json_bytes), C.byref(h))
        if st != 0:
            raise ValueError(f"native tokenizer refused the JSON (status {st})", st)
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            native_lib().czg_tok_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def _error(self, st: int) -> ValueError:
        return ValueError(f"czg_tok error {st}: {native_lib().czg_tok_last_error(self._h).decode()}")

    def encode(self, text: str) -> list[int]:
        b = _utf8(text)
        out = np.empty(max(len(b), 1), np.uint32)
        n = C.c_size_t()
        st = native_lib().czg_tok_encode(self._h, b, len(b), out.ctypes.data, len(out), C.byref(n))
        if st != 0:
            raise self._error(st)
        return out[: n.value].tolist()

    def encode_batch_arrays(self, texts: list[str], num_threads: int = 0) -> list[np.ndarray]:
        bs = [_utf8(t) for t in texts]
        lens = np.array([len(b) for b in bs], np.uint64)
        offs = np.zeros(len(bs), np.uint64)
        if len(bs) > 1:
            offs[1:] = np.cumsum(lens[:-1])
        blob = b"".join(bs)
        buf = C.create_string_buffer(blob, max(len(blob), 1))
        base = C.addressof(buf)
        ptrs = (C.c_void_p * max(len(bs), 1))(*[base + int(o) for o in offs])
        out = np.empty(max(int(lens.sum()), 1), np.uint32)
        n_out = np.zeros(max(len(bs), 1), np.uint64)
        st = native_lib().czg_tok_encode_batch(self._h, len(bs), ptrs, lens.ctypes.data, out.ctypes.data,
                                               offs.ctypes.data, n_out.ctypes.data, int(num_threads))
        if st != 0:
            raise self._error(st)
        return [out[int(o): int(o) + int(k)] for o, k in zip(offs, n_out[: len(bs)])]

    def decode_bytes(self, tokens) -> bytes:
        """Bytes of the tokens; ValueError("Invalid token for decoding: N") as tiktoken.rs:186-198."""
        a64 = np.asarray(tokens, dtype=np.int64).reshape(-1)
        bad = (a64 < 0) | (a64 > 0xFFFFFFFF)
        if bad.any():
            raise ValueError(f"Invalid token for decoding: {int(a64[bad][0])}")
        ids = np.ascontiguousarray(a64.astype(np.uint32))
        n = C.c_size_t()
        L = native_lib()
        st = L.czg_tok_decode(self._h, ids.ctypes.data, len(ids), None, 0, C.byref(n))
        if st != 0:
            raise ValueError(L.czg_tok_last_error(self._h).decode())
        out = C.create_string_buffer(max(n.value, 1))
        st = L.czg_tok_decode(self._h, ids.ctypes.data, len(ids), out, n.value, C.byref(n))
        if st != 0:
            raise self._error(st)
        return out.raw[: n.value]


class Tokenizer:
    def __init__(self, spec: dict, json_bytes: bytes | None = None, native: bool = True):
        ranks = {k.encode("latin-1"): int(v) for k, v in spec["mergeable_ranks"].items()}
        specials = {k: int(v) for k, v in spec["special_tokens"].items()}
        n_vocab = len(ranks) + len(specials)
        explicit = spec.get("explicit_n_vocab")
        if explicit is not None and int(explicit) != n_vocab:
            raise ValueError("explicit_n_vocab != computed size")  # tiktoken.rs:545-548
        self._spec = (spec.get("name", "czm"), spec["pat_str"], ranks, specials, n_vocab)
        self._tiktoken = None
        self.native = None
        if native:
            try:
                self.native = NativeTokenizer(json_bytes if json_bytes is not None
                                              else json.dumps(spec).encode("utf-8"))
            except ValueError as e:
                if len(e.args) < 2 or e.args[1] != E_PATTERN:
                    raise
        self._decoder = {v: k for k, v in ranks.items()}
        self._decoder.update({v: k.encode("utf-8") for k, v in specials.items()})

    def _enc(self):
        """The tiktoken Encoding: the path for other patterns, and a cross-check."""
        if self._tiktoken is None:
            import tiktoken

            name, pat, ranks, specials, n_vocab = self._spec
            self._tiktoken = tiktoken.Encoding(name=name, pat_str=pat, mergeable_ranks=ranks,
                                               special_tokens=specials, explicit_n_vocab=n_vocab)
        return self._tiktoken

    @classmethod
    def from_json_bytes(cls, data: bytes, native: bool = True) -> "Tokenizer":
        return cls(json.loads(data.decode("utf-8")), data, native)

    @classmethod
    def from_model(cls, tokenizer_data: bytes, codec: str, native: bool = True) -> "Tokenizer":
        if codec == "zstd":
            raw = outer_codec.zstd_decompress(tokenizer_data)
        elif codec == "brotli":
            raw = outer_codec.brotli_decompress(tokenizer_data)
        else:
            raise ValueError(f"Unknown tokenizer codec: {codec}")
        return cls.from_json_bytes(raw, native)

    def encode_with_special_tokens(self, text: str) -> list[int]:
        if self.native is not None:
            return self.native.encode(text)
        return self._enc().encode(text, allowed_special="all")

    def encode_batch(self, texts: list[str], num_threads: int = 8) -> list[list[int]]:
        if self.native is not None:
            return [a.tolist() for a in self.native.encode_batch_arrays(texts, num_threads)]
        return self._enc().encode_batch(texts, num_threads=num_threads, allowed_special="all")

    def encode_batch_arrays(self, texts: list[str], num_threads: int = 8) -> list[np.ndarray]:
        """encode_batch with each document's tokens as a uint32 array (no Python lists)."""
        if self.native is not None:
            return self.native.encode_batch_arrays(texts, num_threads)
        return [np.asarray(t, dtype=np.uint32) for t in self.encode_batch(texts, num_threads)]

    def decode_bytes(self, tokens) -> bytes:
        if self.native is not None:
            return self.native.decode_bytes(tokens)
        try:
            return b"".join(self._decoder[int(t)] for t in tokens)
        except KeyError as e:   # tiktoken.rs:186-198
            raise ValueError(f"Invalid token for decoding: {e.args[0]}") from None
