"""CZIPv1 container (rust/src/file_format.rs).

Outer header, 16 bytes (file_format.rs:77-154): magic "CZIPv1", flags u8
(bit 0 multifile), codec_id u8 (0 zstd, 1 brotli), uncompressed_len u32 LE,
header_len u32 LE (inner header size).  Payload = outer-codec(inner header ||
chunk bytes).  Inner header (file_format.rs:158-257): model_id_hash u32,
chunk_count u32, last_chunk_tokens u16, tokenizer_id u8, context_length_log2
u8 (0 reads as 6), then chunk_count u16 byte lengths.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

MAGIC = b"CZIPv1"
OUTER_HEADER_SIZE = 16
DEFAULT_CONTEXT_LENGTH_LOG2 = 6
ZSTD, BROTLI = 0, 1


class FormatError(ValueError):
    pass


@dataclass
class OuterHeader:
    codec_id: int
    uncompressed_len: int
    header_len: int = 0
    flags: int = 0

    def is_multifile(self) -> bool:
        return bool(self.flags & 1)

    def set_multifile(self, v: bool) -> None:
        self.flags = (self.flags | 1) if v else (self.flags & ~1)

    def to_bytes(self) -> bytes:
        return MAGIC + struct.pack("<BBII", self.flags, self.codec_id, self.uncompressed_len,
                                   self.header_len)

    @classmethod
    def from_bytes(cls, data: bytes) -> "OuterHeader":
        if len(data) < OUTER_HEADER_SIZE:
            raise FormatError("Outer header too short")
        if data[:6] != MAGIC:
            raise FormatError(f"Invalid magic bytes: {list(data[:6])}")
        flags, codec, ulen, hlen = struct.unpack_from("<BBII", data, 6)
        if codec not in (ZSTD, BROTLI):
            raise FormatError(f"Unknown codec: {codec}")
        return cls(codec, ulen, hlen, flags)


@dataclass
class InnerHeader:
    model_id_hash: int
    tokenizer_id: int = 0
    context_length_log2: int = DEFAULT_CONTEXT_LENGTH_LOG2
    last_chunk_tokens: int = -1
    chunk_byte_lens: list = field(default_factory=list)

    def __post_init__(self):
        if self.last_chunk_tokens < 0:   # file_format.rs:185-194
            self.last_chunk_tokens = (1 << self.context_length_log2) & 0xFFFF

    @property
    def chunk_count(self) -> int:
        return len(self.chunk_byte_lens)

    def tokens_per_chunk(self) -> int:
        return (1 << self.context_length_log2) & 0xFFFF

    def header_size(self) -> int:
        return 12 + 2 * self.chunk_count

    def to_bytes(self) -> bytes:
        return struct.pack("<IIHBB", self.model_id_hash, self.chunk_count, self.last_chunk_tokens,
                           self.tokenizer_id, self.context_length_log2) + \
            struct.pack(f"<{self.chunk_count}H", *self.chunk_byte_lens)

    @classmethod
    def from_bytes(cls, data: bytes) -> "InnerHeader":
        if len(data) < 12:
            raise FormatError("Inner header too short")
        mh, cc, last, tid, l2 = struct.unpack_from("<IIHBB", data, 0)
        if l2 == 0:
            l2 = DEFAULT_CONTEXT_LENGTH_LOG2
        if len(data) < 12 + 2 * cc:
            raise FormatError(f"Inner header too short for {cc} chunks")
        lens = list(struct.unpack_from(f"<{cc}H", data, 12))
        return cls(mh, tid, l2, last, lens)


@dataclass
class CompressedFile:
    outer: OuterHeader
    inner: InnerHeader
    chunks: list = field(default_factory=list)

    @classmethod
    def with_context_length(cls, model_id_hash: int, tokenizer_id: int, codec: int,
                            uncompressed_len: int, context_length_log2: int) -> "CompressedFile":
        return cls(OuterHeader(codec, uncompressed_len),
                   InnerHeader(model_id_hash, tokenizer_id, context_length_log2))

    def add_chunk(self, data: bytes, is_last: bool, last_chunk_tokens: int) -> None:
        if len(data) > 0xFFFF:   # file_format.rs:311
            raise FormatError("Chunk too large")
        self.inner.chunk_byte_lens.append(len(data))
        if is_last:
            self.inner.last_chunk_tokens = last_chunk_tokens
        self.chunks.append(bytes(data))

    def total_tokens(self) -> int:
        if self.inner.chunk_count == 0:
            return 0
        return (self.inner.chunk_count - 1) * self.inner.tokens_per_chunk() + self.inner.last_chunk_tokens

    def chunk_tokens(self, i: int) -> int:
        if i == self.inner.chunk_count - 1:
            return self.inner.last_chunk_tokens
        return self.inner.tokens_per_chunk()

    def to_bytes_uncompressed(self) -> tuple[bytes, bytes]:
        outer = OuterHeader(self.outer.codec_id, self.outer.uncompressed_len,
                            self.inner.header_size(), self.outer.flags)
        return outer.to_bytes(), self.inner.to_bytes() + b"".join(self.chunks)

    @classmethod
    def read_from_decompressed(cls, outer: OuterHeader, payload: bytes) -> "CompressedFile":
        inner = InnerHeader.from_bytes(payload)
        off = inner.header_size()
        chunks = []
        for n in inner.chunk_byte_lens:
            if len(payload) < off + n:
                raise FormatError("Chunk data truncated")
            chunks.append(payload[off:off + n])
            off += n
        return cls(outer, inner, chunks)
