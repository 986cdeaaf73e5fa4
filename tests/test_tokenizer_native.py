"""The native tokenizer (libczg_tok.so) against the tiktoken package.

tiktoken runs the same algorithm as the reference's CoreBPE (regex split, then
byte-pair merges, specials allowed) through a regex engine of the same family
as the reference's fancy-regex; it is the checker here.  CPU only.
"""
import ctypes as C
import json
import random

import numpy as np
import pytest


@pytest.fixture(scope="module")
def json_bytes(shipped_path):
    from compress_zip_b200 import czm, outer_codec

    mf = czm.ModelFile.load(shipped_path)
    if mf.tokenizer_codec == "zstd":
        return outer_codec.zstd_decompress(mf.tokenizer_data)
    return outer_codec.brotli_decompress(mf.tokenizer_data)


@pytest.fixture(scope="module")
def pair(json_bytes):
    from compress_zip_b200.tokenizer import Tokenizer

    native = Tokenizer.from_json_bytes(json_bytes)
    ref = Tokenizer.from_json_bytes(json_bytes, native=False)
    assert native.native is not None and ref.native is None
    return native, ref


EDGE = [
    "", "a", "'", "'s", "'S", "'ll", "'LL", "'Ve", "'re", "'x", "a'b", " 'x", "'ſ", "ſ's",
    "hello world", "it's I'LL we've they'RE  x", "  leading\n\n  \n trailing   ", "a\r\nb\r\n\r\n",
    "123456 7890 1 22 333 4444", "x<|bos|>y<|eos|>", "<|bos|>", "<|eos|><|bos|>", " <|bos|> ",
    "  \n<|eos|>\n  ", "tab\tsep\t\tend\t", "((a)) !!! ?? ...\n", "café naïve 中文 \U0001F600 emoji",
    "   　 mixed spaces", "end with space ", "\n", "\r", "\r\n", "\n\n\n", "   ", " \n ", "x \n y",
    " word", "\u0085x", "a b", "١٢٣٤", "ⅧⅨ", "½ ¾",
    "x" * 5000, " " * 300 + "y", "ab" * 2000, "<|bos|" + "|>", "<|unknown|>",
]


def test_edge_cases(pair):
    native, ref = pair
    for s in EDGE:
        assert native.encode_with_special_tokens(s) == ref.encode_with_special_tokens(s), repr(s)


def test_random_strings(pair):
    native, ref = pair
    rng = random.Random(1)
    alphabet = [chr(c) for c in list(range(32, 127)) + [9, 10, 11, 12, 13, 0x85, 0xA0, 0xE9, 0x17F, 0x2028,
                                                             0x3000, 0x4E2D, 0x661, 0x2167, 0x1F600, 0x10D4A]]
    for _ in range(4000):
        s = "".join(rng.choice(alphabet) for _ in range(rng.randint(0, 48)))
        assert native.encode_with_special_tokens(s) == ref.encode_with_special_tokens(s), repr(s)


def test_random_unicode(pair):
    """Codepoints from the whole range (no surrogates), so the class tables are exercised."""
    native, ref = pair
    rng = random.Random(2)
    for _ in range(1500):
        cps = []
        for _ in range(rng.randint(1, 24)):
            r = rng.random()
            if r < 0.3:
                cps.append(rng.choice([32, 10, 13, 9, 39, 0x3000]))
            elif r < 0.6:
                cps.append(rng.randint(0x20, 0x2FFF))
            else:
                c = rng.randint(0, 0x10FFFF)
                cps.append(c if not 0xD800 <= c <= 0xDFFF else 0x41)
        s = "".join(map(chr, cps))
        assert native.encode_with_special_tokens(s) == ref.encode_with_special_tokens(s), [hex(c) for c in cps]


def test_documents_and_batch(pair):
    from compress_zip_b200 import synth

    native, ref = pair
    docs = synth.documents(range(40, 52), 6000) + ["", "<|bos|>" + synth.document(3, 500)]
    want = [ref.encode_with_special_tokens(d) for d in docs]
    assert [native.encode_with_special_tokens(d) for d in docs] == want
    assert native.encode_batch(docs, num_threads=4) == want
    assert native.encode_batch(docs, num_threads=1) == want
    assert native.encode_batch([], num_threads=3) == []


def test_decode(pair):
    from compress_zip_b200 import synth

    native, ref = pair
    text = synth.document(9, 2000) + "<|eos|>é中\U0001F600"
    ids = native.encode_with_special_tokens(text)
    assert native.decode_bytes(ids) == text.encode("utf-8") == ref.decode_bytes(ids)
    assert native.decode_bytes([]) == b""
    for bad in ([5000], [-1], [1 << 40]):
        with pytest.raises(ValueError, match="Invalid token for decoding"):
            native.decode_bytes(bad)


def test_lone_surrogates_like_tiktoken(pair):
    native, ref = pair
    s = "ab\ud800cd \udfff"
    assert native.encode_with_special_tokens(s) == ref._enc().encode(s, allowed_special="all")


def test_abi_errors(json_bytes):
    from compress_zip_b200.tokenizer import native_lib

    L = native_lib()
    h = C.c_void_p()
    assert L.czg_tok_create(json_bytes, len(json_bytes), C.byref(h)) == 0
    try:
        out = np.zeros(16, np.uint32)
        n = C.c_size_t()
        assert L.czg_tok_encode(h, b"ab\xff", 3, out.ctypes.data, 16, C.byref(n)) == 5       # invalid UTF-8
        assert L.czg_tok_encode(h, b"\xc0\x80", 2, out.ctypes.data, 16, C.byref(n)) == 5     # overlong
        assert L.czg_tok_encode(h, b"\xed\xa0\x80", 3, out.ctypes.data, 16, C.byref(n)) == 5  # surrogate
        assert L.czg_tok_encode(h, b"hello world", 11, out.ctypes.data, 1, C.byref(n)) == 6   # capacity
        assert n.value >= 2
        assert L.czg_tok_encode(h, b"hello world", 11, None, 0, C.byref(n)) == 0              # size query
        assert L.czg_tok_encode(None, b"x", 1, out.ctypes.data, 16, C.byref(n)) == 1
    finally:
        L.czg_tok_destroy(h)
    bad = json.loads(json_bytes)
    bad["explicit_n_vocab"] = 7
    raw = json.dumps(bad).encode()
    assert L.czg_tok_create(raw, len(raw), C.byref(h)) == 4
    assert L.czg_tok_create(b"{not json", 9, C.byref(h)) == 2


def test_other_pattern_falls_back(json_bytes):
    from compress_zip_b200.tokenizer import Tokenizer

    spec = json.loads(json_bytes)
    spec["pat_str"] = r"\p{L}+|\p{N}+|\s+|[^\s\p{L}\p{N}]+"
    t = Tokenizer(spec)
    assert t.native is None
    assert t.decode_bytes(t.encode_with_special_tokens("abc 12 !!")) == b"abc 12 !!"


def test_merge_kat():
    """tiktoken.rs:566-588: "ab" merges when "ab" is a token, else stays two bytes."""
    from compress_zip_b200.tokenizer import NativeTokenizer, native_lib

    pat = native_lib().czg_tok_pattern().decode()

    def spec(with_ab):
        ranks = {chr(b): b for b in range(256)}
        if with_ab:
            ranks["ab"] = 256
        return json.dumps({"pat_str": pat, "mergeable_ranks": ranks, "special_tokens": {}}).encode()

    assert NativeTokenizer(spec(True)).encode("ab") == [256]
    assert NativeTokenizer(spec(False)).encode("ab") == [97, 98]


def test_class_tables_match_engine(root):
    """unicode_classes.inc is what its generator reads off the tiktoken regex engine now."""
    import importlib.util
    import os

    gen = os.path.join(root, "compress-zip_b200", "csrc", "gen_unicode_classes.py")
    spec = importlib.util.spec_from_file_location("gen_unicode_classes", gen)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    inc = open(os.path.join(root, "compress-zip_b200", "csrc", "unicode_classes.inc")).read()
    for name, pat in (("kLetter", r"\p{L}"), ("kNumber", r"\p{N}"), ("kSpace", r"\s")):
        rs = m.ranges(m.members(pat))
        body = inc.split(f"static const uint32_t {name}[][2] = {{")[1].split("};")[0]
        got = [tuple(int(x, 16) for x in pr.strip("{} ").split(", ")) for pr in body.replace("\n", " ").split("},") if "0x" in pr]
        assert got == rs, name


def test_exports(root):
    import os
    import re

    from compress_zip_b200.tokenizer import native_lib

    L = native_lib()
    hdr = open(os.path.join(root, "include", "czg_tok.h")).read()
    names = set(re.findall(r"\b(czg_tok_\w+)\s*\(", hdr))
    assert names >= {"czg_tok_create", "czg_tok_encode", "czg_tok_encode_batch", "czg_tok_decode"}
    for n in names:
        assert hasattr(L, n), n
