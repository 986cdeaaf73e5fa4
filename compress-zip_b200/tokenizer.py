"""BPE tokenizer of a .czm model (host pre/post step, outside the GPU path).

The reference embeds a zstd- or brotli-compressed tiktoken JSON in the model
(``tokenizer.data``, decoded at rust/src/main.rs:88-109 and 157-163) and
encodes with special tokens allowed (rust/src/tiktoken.rs:498-501).  JSON keys
map one codepoint to one byte (tiktoken.rs:517-527).  The same BPE algorithm
is run here through the ``tiktoken`` package.
"""
from __future__ import annotations

import json

from . import outer_codec


class Tokenizer:
    def __init__(self, spec: dict):
        import tiktoken

        ranks = {k.encode("latin-1"): int(v) for k, v in spec["mergeable_ranks"].items()}
        specials = {k: int(v) for k, v in spec["special_tokens"].items()}
        n_vocab = len(ranks) + len(specials)
        explicit = spec.get("explicit_n_vocab")
        if explicit is not None and int(explicit) != n_vocab:
            raise ValueError("explicit_n_vocab != computed size")  # tiktoken.rs:545-548
        self._enc = tiktoken.Encoding(
            name=spec.get("name", "czm"), pat_str=spec["pat_str"],
            mergeable_ranks=ranks, special_tokens=specials, explicit_n_vocab=n_vocab)
        self._decoder = {v: k for k, v in ranks.items()}
        self._decoder.update({v: k.encode("utf-8") for k, v in specials.items()})

    @classmethod
    def from_json_bytes(cls, data: bytes) -> "Tokenizer":
        return cls(json.loads(data.decode("utf-8")))

    @classmethod
    def from_model(cls, tokenizer_data: bytes, codec: str) -> "Tokenizer":
        if codec == "zstd":
            raw = outer_codec.zstd_decompress(tokenizer_data)
        elif codec == "brotli":
            raw = outer_codec.brotli_decompress(tokenizer_data)
        else:
            raise ValueError(f"Unknown tokenizer codec: {codec}")
        return cls.from_json_bytes(raw)

    def encode_with_special_tokens(self, text: str) -> list[int]:
        return self._enc.encode(text, allowed_special="all")

    def encode_batch(self, texts: list[str], num_threads: int = 8) -> list[list[int]]:
        return self._enc.encode_batch(texts, num_threads=num_threads, allowed_special="all")

    def decode_bytes(self, tokens) -> bytes:
        try:
            return b"".join(self._decoder[int(t)] for t in tokens)
        except KeyError as e:   # tiktoken.rs:186-198
            raise ValueError(f"Invalid token for decoding: {e.args[0]}") from None
