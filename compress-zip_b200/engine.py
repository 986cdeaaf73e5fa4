"""ctypes binding of the C ABI in include/czg.h (libczg.so, CUDA for sm_100a).

This is the GPU path: there is no CPU fallback.  If libczg.so is missing or no
CUDA device is present, constructing an Engine raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libczg.so")

CZG_OK = 0
STATUS_NAMES = {1: "CZG_E_ARG", 2: "CZG_E_MODEL", 3: "CZG_E_UNSUPPORTED", 4: "CZG_E_CAPACITY",
                5: "CZG_E_DEVICE", 6: "CZG_E_TIMEOUT", 7: "CZG_E_TOKEN", 8: "CZG_E_CHUNK",
                9: "CZG_E_LIMIT"}
MAX_KERNEL_CLASSES = 24

# The exported symbols of include/czg.h, checked by the CPU test suite.
EXPORTS = ["czg_ctx_create", "czg_ctx_destroy", "czg_last_error", "czg_model_info_get",
           "czg_compress_bound", "czg_compress_chunks", "czg_compress_chunks_device",
           "czg_decompress_chunks", "czg_last_stats", "czg_kernel_name", "czg_debug_trace",
           "czg_set_stream", "czg_encode_intervals_static", "czg_set_kernel_timing",
           "czg_debug_encode_intervals"]


class CzgError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("vocab_size", "n_layers", "n_heads", "n_kv_heads",
                                         "d_model", "d_ff", "head_dim", "max_seq_len",
                                         "context_length")] + \
               [("coef_q24", C.c_uint32), ("target_total", C.c_uint32)]


class Stats(C.Structure):
    _fields_ = [("total_ms", C.c_double), ("h2d_ms", C.c_double), ("d2h_ms", C.c_double),
                ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64),
                ("n_tokens", C.c_uint64), ("n_chunks", C.c_uint64), ("n_classes", C.c_uint32),
                ("kernel_ms", C.c_double * MAX_KERNEL_CLASSES),
                ("launches", C.c_uint64 * MAX_KERNEL_CLASSES)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built (run compress-zip_b200/build.py); "
                               "the GPU path has no fallback")
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        L.czg_ctx_create.argtypes = [C.c_int, P, C.c_size_t, C.POINTER(P)]
        L.czg_ctx_create.restype = C.c_int
        L.czg_ctx_destroy.argtypes = [P]
        L.czg_ctx_destroy.restype = None
        L.czg_last_error.argtypes = [P]
        L.czg_last_error.restype = C.c_char_p
        L.czg_model_info_get.argtypes = [P, C.POINTER(ModelInfo)]
        L.czg_compress_bound.argtypes = [C.c_uint64, C.c_uint64]
        L.czg_compress_bound.restype = C.c_uint64
        for fn in (L.czg_compress_chunks, L.czg_compress_chunks_device):
            fn.argtypes = [P, P, P, C.c_uint32, P, C.c_uint64, P, C.POINTER(C.c_uint64)]
            fn.restype = C.c_int
        L.czg_decompress_chunks.argtypes = [P, P, P, P, C.c_uint32, P]
        L.czg_decompress_chunks.restype = C.c_int
        L.czg_last_stats.argtypes = [P, C.POINTER(Stats)]
        L.czg_kernel_name.argtypes = [C.c_uint32]
        L.czg_kernel_name.restype = C.c_char_p
        L.czg_debug_trace.argtypes = [P, P, C.c_uint32, P, P, P, P]
        L.czg_debug_trace.restype = C.c_int
        L.czg_set_stream.argtypes = [P, P]
        L.czg_set_stream.restype = C.c_int
        L.czg_set_kernel_timing.argtypes = [P, C.c_int]
        L.czg_set_kernel_timing.restype = C.c_int
        L.czg_encode_intervals_static.argtypes = [P, P, C.c_uint32, C.c_uint64, C.c_uint32, P,
                                                   C.c_uint64, P, C.POINTER(C.c_uint64), P]
        L.czg_encode_intervals_static.restype = C.c_int
        L.czg_debug_encode_intervals.argtypes = [P, P, P, C.c_uint32, P, C.c_uint64, P, C.POINTER(C.c_uint64)]
        L.czg_debug_encode_intervals.restype = C.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class Engine:
    """One context on one device: the model weights plus a wave workspace."""

    def __init__(self, model_bytes: bytes, device: int = 0):
        L = lib()
        self._buf = np.frombuffer(model_bytes, dtype=np.uint8)
        h = C.c_void_p()
        st = L.czg_ctx_create(device, _p(self._buf), len(self._buf), C.byref(h))
        if st != CZG_OK:
            raise CzgError(st, L.czg_last_error(None).decode())
        self._h = h
        self.device = device
        mi = ModelInfo()
        L.czg_model_info_get(h, C.byref(mi))
        self.info = {k: getattr(mi, k) for k, _ in ModelInfo._fields_}

    @classmethod
    def from_file(cls, path: str, device: int = 0) -> "Engine":
        with open(path, "rb") as f:
            return cls(f.read(), device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().czg_ctx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int) -> None:
        if st != CZG_OK:
            raise CzgError(st, lib().czg_last_error(self._h).decode())

    # ---- compress ------------------------------------------------------------
    def compress_packed(self, tokens: np.ndarray, chunk_starts: np.ndarray,
                        out: np.ndarray | None = None):
        """Returns (packed bytes array, per-chunk lengths)."""
        L = lib()
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        starts = np.ascontiguousarray(chunk_starts, dtype=np.uint64)
        n = len(starts) - 1
        lens = np.zeros(max(n, 1), dtype=np.uint32)
        need = C.c_uint64(0)
        bound = L.czg_compress_bound(int(starts[-1] - starts[0]) if n > 0 else 0, max(n, 0))
        if out is None or len(out) < bound:
            out = np.empty(max(bound, 1), dtype=np.uint8)
        if n <= 0:
            return out[:0], lens[:0]
        self._check(L.czg_compress_chunks(self._h, _p(tokens), _p(starts), n, _p(out), len(out),
                                          _p(lens), C.byref(need)))
        return out[: need.value], lens[:n]

    def compress_chunks(self, tokens: np.ndarray, chunk_starts: np.ndarray) -> list[bytes]:
        packed, lens = self.compress_packed(tokens, chunk_starts)
        offs = np.concatenate([[0], np.cumsum(lens, dtype=np.uint64)]).astype(np.int64)
        raw = packed.tobytes()
        return [raw[offs[i]:offs[i + 1]] for i in range(len(lens))]

    def compress_device(self, d_tokens_ptr: int, chunk_starts: np.ndarray, out: np.ndarray,
                        lens: np.ndarray) -> int:
        """Tokens already in device memory; returns the packed byte count."""
        starts = np.ascontiguousarray(chunk_starts, dtype=np.uint64)
        n = len(starts) - 1
        need = C.c_uint64(0)
        self._check(lib().czg_compress_chunks_device(self._h, C.c_void_p(d_tokens_ptr), _p(starts),
                                                     n, _p(out), len(out), _p(lens),
                                                     C.byref(need)))
        return need.value

    # ---- decompress ----------------------------------------------------------
    def decompress_chunks(self, chunks: list[bytes], n_tokens, out: np.ndarray | None = None) -> np.ndarray:
        """Tokens of every chunk, chunk after chunk.  ``out`` (optional): a contiguous
        uint32 buffer of at least sum(n_tokens) entries to decode into, reused across
        calls (a fresh buffer's pages are first touched by the copy); the result is a
        view of it."""
        n = len(chunks)
        nt = np.ascontiguousarray(n_tokens, dtype=np.uint32)
        total = int(nt.sum(dtype=np.uint64))
        if out is None:   # every token of every chunk is written by the call (no zero fill needed)
            out = np.empty(max(total, 1), dtype=np.uint32)
        elif out.dtype != np.uint32 or not out.flags["C_CONTIGUOUS"] or out.ndim != 1 or len(out) < max(total, 1):
            raise ValueError("out must be a contiguous 1-D uint32 array of at least sum(n_tokens) entries")
        if n == 0:
            return out[:0]
        data = np.frombuffer(b"".join(chunks) or b"\0", dtype=np.uint8)   # read only
        starts = np.zeros(n + 1, dtype=np.uint64)
        np.cumsum(np.fromiter(map(len, chunks), dtype=np.uint64, count=n), out=starts[1:])
        self._check(lib().czg_decompress_chunks(self._h, _p(data), _p(starts), _p(nt), n, _p(out)))
        return out[:total]

    def set_stream(self, stream_handle: int | None) -> None:
        """Run subsequent work on a caller's cudaStream_t (None: the own stream)."""
        self._check(lib().czg_set_stream(self._h, C.c_void_p(stream_handle or 0)))

    def set_kernel_timing(self, on: bool) -> None:
        """Time every kernel with CUDA events (last_stats()['kernels']); off by default."""
        self._check(lib().czg_set_kernel_timing(self._h, int(bool(on))))

    # ---- diagnostics -----------------------------------------------------------
    def last_stats(self) -> dict:
        L = lib()
        s = Stats()
        L.czg_last_stats(self._h, C.byref(s))
        kernels = {}
        for i in range(s.n_classes):
            kernels[L.czg_kernel_name(i).decode()] = {"ms": s.kernel_ms[i],
                                                      "launches": int(s.launches[i])}
        return {"total_ms": s.total_ms, "h2d_ms": s.h2d_ms, "d2h_ms": s.d2h_ms,
                "h2d_bytes": int(s.h2d_bytes), "d2h_bytes": int(s.d2h_bytes),
                "n_tokens": int(s.n_tokens), "n_chunks": int(s.n_chunks), "kernels": kernels}

    def debug_trace(self, tokens: np.ndarray) -> dict:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = len(tokens)
        V, d, nl = self.info["vocab_size"], self.info["d_model"], self.info["n_layers"]
        logits = np.zeros((n, V), dtype=np.int32)
        lohi = np.zeros((n, 2), dtype=np.uint32)
        attn = np.zeros((n, nl, d), dtype=np.int8)
        fin = np.zeros((n, d), dtype=np.int8)
        self._check(lib().czg_debug_trace(self._h, _p(tokens), n, _p(logits), _p(lohi), _p(attn),
                                          _p(fin)))
        return {"logits": logits, "lohi": lohi, "attn": attn, "final_in": fin}

    def debug_encode_intervals(self, lohi: np.ndarray, chunk_starts: np.ndarray) -> list[bytes]:
        """The compress path's encoder alone on given (sym_low, sym_high) pairs."""
        lohi = np.ascontiguousarray(lohi, dtype=np.uint32).reshape(-1, 2)
        starts = np.ascontiguousarray(chunk_starts, dtype=np.uint64)
        n = len(starts) - 1
        if n <= 0:
            return []
        lens = np.zeros(n, dtype=np.uint32)
        out = np.empty(max(4 * len(lohi) + 8 * n, 1), dtype=np.uint8)
        need = C.c_uint64(0)
        self._check(lib().czg_debug_encode_intervals(self._h, _p(lohi), _p(starts), n, _p(out), len(out),
                                                     _p(lens), C.byref(need)))
        offs = np.concatenate([[0], np.cumsum(lens, dtype=np.uint64)]).astype(np.int64)
        raw = out[: need.value].tobytes()
        return [raw[offs[i]:offs[i + 1]] for i in range(n)]
