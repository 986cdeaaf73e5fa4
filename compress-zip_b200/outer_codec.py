"""Outer codec of the CZIPv1 container: zstd level 22 or brotli q11/lgwin22.

The reference calls the Rust crates ``zstd`` 0.13.3 (zstd-sys 2.0.16+zstd.1.5.7)
and ``brotli`` 6.0.0 at rust/src/main.rs:261-275 (compress) and 348-359
(decompress).  This host step stays on the CPU.  Here it is driven through the
system C libraries (libzstd.so.1, libbrotlienc/dec.so.1) with the same call
shapes as the Rust side:

* zstd: a streaming encoder at level 22 with no pledged source size, as
  ``zstd::encode_all`` does (so the frame header carries no content size);
* brotli: an encoder instance with quality 11 and lgwin 22, all input given in
  PROCESS operations and then FINISH, as ``brotli::CompressorWriter`` does.
"""
from __future__ import annotations

import ctypes as C
import ctypes.util

ZSTD = 0
BROTLI = 1

_zstd = None
_benc = None
_bdec = None


def _load(names):
    for n in names:
        try:
            return C.CDLL(n)
        except OSError:
            continue
    raise OSError(f"none of {names} could be loaded")


def _z():
    global _zstd
    if _zstd is None:
        L = _load(["libzstd.so.1", ctypes.util.find_library("zstd") or "libzstd.so"])
        L.ZSTD_createCCtx.restype = C.c_void_p
        L.ZSTD_freeCCtx.argtypes = [C.c_void_p]
        L.ZSTD_CCtx_setParameter.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.ZSTD_CCtx_setParameter.restype = C.c_size_t
        L.ZSTD_compressStream2.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.ZSTD_compressStream2.restype = C.c_size_t
        L.ZSTD_isError.argtypes = [C.c_size_t]
        L.ZSTD_isError.restype = C.c_uint
        L.ZSTD_getErrorName.argtypes = [C.c_size_t]
        L.ZSTD_getErrorName.restype = C.c_char_p
        L.ZSTD_CStreamOutSize.restype = C.c_size_t
        L.ZSTD_createDCtx.restype = C.c_void_p
        L.ZSTD_freeDCtx.argtypes = [C.c_void_p]
        L.ZSTD_decompressStream.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.ZSTD_decompressStream.restype = C.c_size_t
        L.ZSTD_DStreamOutSize.restype = C.c_size_t
        _zstd = L
    return _zstd


class _ZBuf(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("size", C.c_size_t), ("pos", C.c_size_t)]


def zstd_compress(data: bytes, level: int = 22) -> bytes:
    L = _z()
    cctx = L.ZSTD_createCCtx()
    try:
        L.ZSTD_CCtx_setParameter(cctx, 100, level)  # ZSTD_c_compressionLevel
        src = C.create_string_buffer(data, len(data))
        inb = _ZBuf(C.cast(src, C.c_void_p), len(data), 0)
        cap = L.ZSTD_CStreamOutSize()
        dst = C.create_string_buffer(cap)
        out = bytearray()
        while True:
            outb = _ZBuf(C.cast(dst, C.c_void_p), cap, 0)
            mode = 0 if inb.pos < inb.size else 2  # ZSTD_e_continue, then ZSTD_e_end
            r = L.ZSTD_compressStream2(cctx, C.byref(outb), C.byref(inb), mode)
            if L.ZSTD_isError(r):
                raise ValueError("zstd: " + L.ZSTD_getErrorName(r).decode())
            out += dst.raw[: outb.pos]
            if mode == 2 and r == 0:
                break
        return bytes(out)
    finally:
        L.ZSTD_freeCCtx(cctx)


def zstd_decompress(data: bytes) -> bytes:
    L = _z()
    dctx = L.ZSTD_createDCtx()
    try:
        src = C.create_string_buffer(data, len(data))
        inb = _ZBuf(C.cast(src, C.c_void_p), len(data), 0)
        cap = L.ZSTD_DStreamOutSize()
        dst = C.create_string_buffer(cap)
        out = bytearray()
        while True:
            outb = _ZBuf(C.cast(dst, C.c_void_p), cap, 0)
            r = L.ZSTD_decompressStream(dctx, C.byref(outb), C.byref(inb))
            if L.ZSTD_isError(r):
                raise ValueError("zstd: " + L.ZSTD_getErrorName(r).decode())
            out += dst.raw[: outb.pos]
            if inb.pos >= inb.size and outb.pos < cap:
                if r != 0:
                    raise ValueError("zstd: truncated frame")
                break
        return bytes(out)
    finally:
        L.ZSTD_freeDCtx(dctx)


def _be():
    global _benc
    if _benc is None:
        L = _load(["libbrotlienc.so.1", ctypes.util.find_library("brotlienc") or "libbrotlienc.so"])
        L.BrotliEncoderCreateInstance.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.BrotliEncoderCreateInstance.restype = C.c_void_p
        L.BrotliEncoderSetParameter.argtypes = [C.c_void_p, C.c_int, C.c_uint32]
        L.BrotliEncoderSetParameter.restype = C.c_int
        L.BrotliEncoderCompressStream.argtypes = [
            C.c_void_p, C.c_int, C.POINTER(C.c_size_t), C.POINTER(C.c_void_p),
            C.POINTER(C.c_size_t), C.POINTER(C.c_void_p), C.c_void_p]
        L.BrotliEncoderCompressStream.restype = C.c_int
        L.BrotliEncoderIsFinished.argtypes = [C.c_void_p]
        L.BrotliEncoderIsFinished.restype = C.c_int
        L.BrotliEncoderDestroyInstance.argtypes = [C.c_void_p]
        _benc = L
    return _benc


def _bd():
    global _bdec
    if _bdec is None:
        L = _load(["libbrotlidec.so.1", ctypes.util.find_library("brotlidec") or "libbrotlidec.so"])
        L.BrotliDecoderCreateInstance.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        L.BrotliDecoderCreateInstance.restype = C.c_void_p
        L.BrotliDecoderDecompressStream.argtypes = [
            C.c_void_p, C.POINTER(C.c_size_t), C.POINTER(C.c_void_p),
            C.POINTER(C.c_size_t), C.POINTER(C.c_void_p), C.c_void_p]
        L.BrotliDecoderDecompressStream.restype = C.c_int
        L.BrotliDecoderDestroyInstance.argtypes = [C.c_void_p]
        _bdec = L
    return _bdec


def brotli_compress(data: bytes, quality: int = 11, lgwin: int = 22) -> bytes:
    L = _be()
    st = L.BrotliEncoderCreateInstance(None, None, None)
    try:
        L.BrotliEncoderSetParameter(st, 1, quality)  # BROTLI_PARAM_QUALITY
        L.BrotliEncoderSetParameter(st, 2, lgwin)    # BROTLI_PARAM_LGWIN
        src = C.create_string_buffer(data, len(data))
        avail_in = C.c_size_t(len(data))
        next_in = C.c_void_p(C.cast(src, C.c_void_p).value)
        cap = 4096
        dst = C.create_string_buffer(cap)
        out = bytearray()
        op = 0  # BROTLI_OPERATION_PROCESS until all input is taken, then FINISH (2)
        while True:
            if op == 0 and avail_in.value == 0:
                op = 2
            avail_out = C.c_size_t(cap)
            next_out = C.c_void_p(C.cast(dst, C.c_void_p).value)
            if not L.BrotliEncoderCompressStream(st, op, C.byref(avail_in), C.byref(next_in),
                                                 C.byref(avail_out), C.byref(next_out), None):
                raise ValueError("brotli encoder error")
            out += dst.raw[: cap - avail_out.value]
            if op == 2 and L.BrotliEncoderIsFinished(st):
                break
        return bytes(out)
    finally:
        L.BrotliEncoderDestroyInstance(st)


def brotli_decompress(data: bytes) -> bytes:
    L = _bd()
    st = L.BrotliDecoderCreateInstance(None, None, None)
    try:
        src = C.create_string_buffer(data, len(data))
        avail_in = C.c_size_t(len(data))
        next_in = C.c_void_p(C.cast(src, C.c_void_p).value)
        cap = 1 << 16
        dst = C.create_string_buffer(cap)
        out = bytearray()
        while True:
            avail_out = C.c_size_t(cap)
            next_out = C.c_void_p(C.cast(dst, C.c_void_p).value)
            r = L.BrotliDecoderDecompressStream(st, C.byref(avail_in), C.byref(next_in),
                                                C.byref(avail_out), C.byref(next_out), None)
            out += dst.raw[: cap - avail_out.value]
            if r == 1:      # BROTLI_DECODER_RESULT_SUCCESS
                return bytes(out)
            if r == 3:      # NEEDS_MORE_OUTPUT
                continue
            raise ValueError("brotli: corrupt or truncated stream")
    finally:
        L.BrotliDecoderDestroyInstance(st)


def compress(data: bytes, codec: int) -> bytes:
    if codec == ZSTD:
        return zstd_compress(data, 22)
    if codec == BROTLI:
        return brotli_compress(data, 11, 22)
    raise ValueError(f"Unknown codec: {codec}")


def decompress(data: bytes, codec: int) -> bytes:
    if codec == ZSTD:
        return zstd_decompress(data)
    if codec == BROTLI:
        return brotli_decompress(data)
    raise ValueError(f"Unknown codec: {codec}")
