"""ctypes front end of the CPU oracle (oracle/czoracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by bench.py's CPU-baseline / reference arm, always as the checker or the
CPU baseline, never as the product path.

The .czm is read here with the independent ``safetensors`` package (not with
the product's own parser), following the metadata defaults and tensor names of
the reference loader, rust/src/model.rs:108-274.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATHS = {"generic": os.path.join(_HERE, "libczoracle.so"),
              "avx2": os.path.join(_HERE, "libczoracle_avx2.so")}
MAX_LAYERS = 64
BOS = 1022


def build() -> str:
    """Compile the oracle with its Makefile (checker build, not the product)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATHS["generic"]


_libs: dict = {}


def lib(variant: str = "generic") -> C.CDLL:
    """The oracle library: "generic" (default x86-64 target) or "avx2" (x86-64-v3)."""
    if variant not in _libs:
        path = _LIB_PATHS[variant]
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        _declare(L)
        _libs[variant] = L
    return _libs[variant]


class Layer(C.Structure):
    _fields_ = [
        ("attn_norm", C.c_void_p), ("post_attn_norm", C.c_void_p),
        ("ffn_norm", C.c_void_p), ("post_ffn_norm", C.c_void_p),
        ("qkv_w", C.c_void_p), ("out_w", C.c_void_p), ("up_w", C.c_void_p),
        ("down_w", C.c_void_p), ("score_mult", C.c_void_p), ("sink_key", C.c_void_p),
        ("qkv_mult", C.c_int32), ("out_mult", C.c_int32), ("up_mult", C.c_int32),
        ("down_mult", C.c_int32),
        ("qkv_shift", C.c_int32), ("out_shift", C.c_int32), ("up_shift", C.c_int32),
        ("down_shift", C.c_int32),
    ]


class Model(C.Structure):
    _fields_ = [
        ("vocab", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32), ("d_model", C.c_int32), ("d_ff", C.c_int32),
        ("head_dim", C.c_int32), ("max_seq_len", C.c_int32), ("context_length", C.c_int32),
        ("coef_q24", C.c_uint32), ("target_total", C.c_uint32), ("eps_scaled", C.c_int32),
        ("embed", C.c_void_p), ("final_norm", C.c_void_p), ("head_w", C.c_void_p),
        ("exp2_lut", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("layers", Layer * MAX_LAYERS),
    ]


class Encoder(C.Structure):
    _fields_ = [
        ("low", C.c_uint64), ("high", C.c_uint64), ("underflow", C.c_uint32),
        ("out", C.c_void_p), ("len", C.c_size_t), ("cap", C.c_size_t),
        ("cur", C.c_uint8), ("bit_pos", C.c_int), ("overflow", C.c_int),
    ]


class Decoder(C.Structure):
    _fields_ = [
        ("low", C.c_uint64), ("high", C.c_uint64), ("code", C.c_uint64),
        ("inp", C.c_void_p), ("len", C.c_size_t), ("byte_pos", C.c_size_t),
        ("bit_pos", C.c_int),
    ]


def _declare(L: C.CDLL) -> None:
    P = C.c_void_p
    sig = {
        "czo_clamp_i8": (C.c_int8, [C.c_int32]),
        "czo_sra_rne_s32": (C.c_int32, [C.c_int32, C.c_uint32]),
        "czo_sra_rne_s64_to_s32": (C.c_int32, [C.c_int64, C.c_uint32]),
        "czo_udiv_rne_u32": (C.c_uint32, [C.c_uint32, C.c_uint32]),
        "czo_div_rne_s32_by_u64": (C.c_int32, [C.c_int32, C.c_uint64]),
        "czo_isqrt32": (C.c_uint32, [C.c_uint32]),
        "czo_exp_q16": (C.c_uint16, [C.c_int32, P, C.c_uint32]),
        "czo_inv_rms_q15": (C.c_int32, [C.c_int32]),
        "czo_rmsnorm_i8": (None, [P, P, C.c_int, C.c_int32, P]),
        "czo_linear_i8_i32": (None, [P, P, C.c_int, C.c_int, P]),
        "czo_requant": (None, [P, C.c_int, C.c_int32, C.c_int8, P]),
        "czo_reglu": (None, [P, C.c_int, P]),
        "czo_rope_k": (None, [P, P, P, C.c_int]),
        "czo_rope_q": (None, [P, P, P, C.c_int]),
        "czo_attn_coef_q24": (C.c_uint32, []),
        "czo_build_cumfreqs": (None, [P, C.c_int, P, C.c_uint32, C.c_uint32, P]),
        "czo_default_coef_q24": (C.c_uint32, []),
        "czo_default_target_total": (C.c_uint32, [C.c_int]),
        "czo_model_check": (C.c_int, [P]),
        "czo_kv_bytes": (C.c_size_t, [P]),
        "czo_forward": (None, [P, P, C.c_uint32, C.c_int, P]),
        "czo_enc_init": (None, [P, P, C.c_size_t]),
        "czo_enc_encode": (None, [P, P, C.c_int, C.c_int]),
        "czo_enc_encode_range": (None, [P, C.c_uint32, C.c_uint32, C.c_uint32]),
        "czo_enc_finish": (None, [P]),
        "czo_dec_init": (None, [P, P, C.c_size_t]),
        "czo_dec_decode": (C.c_int, [P, P, C.c_int]),
        "czo_compress_chunks": (C.c_int, [P, P, P, C.c_uint32, P, C.c_uint64, P, C.c_int]),
        "czo_decompress_chunks": (C.c_int, [P, P, P, P, C.c_uint32, P, C.c_int]),
        "czo_chunk_trace": (None, [P, P, C.c_int, P, P, P, P]),
        "czo_attention_seq": (None, [P, P, P, C.c_int, C.c_int, P, P, P, P, P, P]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------------------
# model loading (rust/src/model.rs:108-274, metadata defaults 113-145)
# ---------------------------------------------------------------------------
class OracleModel:
    """A .czm model held as numpy arrays plus the C struct that points at them."""

    def __init__(self, tensors: dict, metadata: dict):
        self.tensors = {k: np.ascontiguousarray(v) for k, v in tensors.items()}
        md = metadata or {}

        def pu(key, default):
            try:
                return int(md[key])
            except (KeyError, ValueError):
                return default

        if "context_length" in md and md["context_length"].isdigit():
            ctx = int(md["context_length"])
        elif "context_length_log2" in md and md["context_length_log2"].isdigit():
            ctx = 1 << int(md["context_length_log2"])
        else:
            ctx = pu("max_seq_len", 64)
        self.cfg = dict(
            vocab_size=pu("vocab_size", 1024), n_layers=pu("n_layers", 1),
            n_heads=pu("n_heads", 6), n_kv_heads=pu("n_kv_heads", 1),
            d_model=pu("d_model", 384), d_ff=pu("d_ff", 1024), head_dim=pu("head_dim", 64),
            max_seq_len=pu("max_seq_len", 64), context_length=ctx,
        )
        t = self.tensors
        m = Model()
        c = self.cfg
        m.vocab, m.n_layers, m.n_heads = c["vocab_size"], c["n_layers"], c["n_heads"]
        m.n_kv_heads, m.d_model, m.d_ff = c["n_kv_heads"], c["d_model"], c["d_ff"]
        m.head_dim, m.max_seq_len, m.context_length = c["head_dim"], c["max_seq_len"], ctx
        L = lib()
        m.coef_q24 = int(t["softmax.coef_q24"].reshape(-1)[0]) if "softmax.coef_q24" in t \
            else L.czo_default_coef_q24()
        m.target_total = int(t["softmax.target_total"].reshape(-1)[0]) \
            if "softmax.target_total" in t else L.czo_default_target_total(m.vocab)
        m.eps_scaled = 1  # rmsnorm.rs:80-83 with eps 1e-5
        m.embed = ptr(t["embed.weight"])
        m.final_norm = ptr(t["norm.weight"])
        m.head_w = ptr(t["head.weight"])
        m.exp2_lut = ptr(t["lut.exp2"])
        m.rope_cos = ptr(t["lut.rope_cos"])
        m.rope_sin = ptr(t["lut.rope_sin"])

        def scalar(name, default):
            return int(t[name].reshape(-1)[0]) if name in t else default

        for i in range(m.n_layers):
            p = f"layers.{i}."
            ly = m.layers[i]
            ly.attn_norm = ptr(t[p + "attn_norm.weight"])
            ly.post_attn_norm = ptr(t[p + "post_attn_norm.weight"])
            ly.ffn_norm = ptr(t[p + "ffn_norm.weight"])
            ly.post_ffn_norm = ptr(t[p + "post_ffn_norm.weight"])
            ly.qkv_w = ptr(t[p + "attn.qkv.weight"])
            ly.out_w = ptr(t[p + "attn.out.weight"])
            ly.up_w = ptr(t[p + "ffn.up.weight"])
            ly.down_w = ptr(t[p + "ffn.down.weight"])
            ly.score_mult = ptr(t[p + "attn.score_mult"])
            ly.sink_key = ptr(t[p + "attn.sink_key"]) if (p + "attn.sink_key") in t else None
            # model.rs:157-170: a missing mult reads as 1, a missing shift as 0
            ly.qkv_mult = scalar(p + "attn.qkv.mult", 1)
            ly.out_mult = scalar(p + "attn.out.mult", 1)
            ly.up_mult = scalar(p + "ffn.up.mult", 1)
            ly.down_mult = scalar(p + "ffn.down.mult", 1)
            ly.qkv_shift = scalar(p + "attn.qkv.shift", 0)
            ly.out_shift = scalar(p + "attn.out.shift", 0)
            ly.up_shift = scalar(p + "ffn.up.shift", 0)
            ly.down_shift = scalar(p + "ffn.down.shift", 0)
        self.struct = m
        self.vocab = m.vocab
        self.d_model = m.d_model
        self.n_layers = m.n_layers

    @property
    def ref(self):
        return C.byref(self.struct)

    def check(self) -> int:
        return lib().czo_model_check(self.ref)

    @property
    def coef_q24(self) -> int:
        return self.struct.coef_q24

    @property
    def target_total(self) -> int:
        return self.struct.target_total


def load_model(path: str) -> OracleModel:
    from safetensors import safe_open

    with safe_open(path, "np") as f:
        md = f.metadata()
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    return OracleModel(tensors, md)


# ---------------------------------------------------------------------------
# chunk drivers and traces
# ---------------------------------------------------------------------------
def slot_cap(n_tokens: int) -> int:
    """Bytes one chunk can need: at most 32 renormalisation bits per symbol
    plus the terminating bit."""
    return 4 * n_tokens + 8


def compress_chunks(model: OracleModel, tokens: np.ndarray, chunk_starts: np.ndarray,
                    nthreads: int | None = None, variant: str = "generic") -> list[bytes]:
    tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
    starts = np.ascontiguousarray(chunk_starts, dtype=np.uint64)
    n = len(starts) - 1
    if n <= 0:
        return []
    cap = slot_cap(int(np.max(np.diff(starts))))
    out = np.zeros(n * cap, dtype=np.uint8)
    lens = np.zeros(n, dtype=np.uint32)
    nt = nthreads or os.cpu_count() or 1
    st = lib(variant).czo_compress_chunks(model.ref, ptr(tokens), ptr(starts), n, ptr(out), cap,
                                          ptr(lens), nt)
    if st != 0:
        raise ValueError(f"oracle compress failed ({st})")
    return [out[i * cap: i * cap + int(lens[i])].tobytes() for i in range(n)]


def decompress_chunks(model: OracleModel, chunks: list[bytes], n_tokens,
                      nthreads: int | None = None, variant: str = "generic") -> np.ndarray:
    n = len(chunks)
    if n == 0:
        return np.zeros(0, dtype=np.uint32)
    data = np.frombuffer(b"".join(chunks) + b"\0", dtype=np.uint8).copy()
    starts = np.zeros(n + 1, dtype=np.uint64)
    starts[1:] = np.cumsum([len(c) for c in chunks])
    nt_arr = np.ascontiguousarray(n_tokens, dtype=np.uint32)
    out = np.zeros(int(nt_arr.sum()), dtype=np.uint32)
    st = lib(variant).czo_decompress_chunks(model.ref, ptr(data), ptr(starts), ptr(nt_arr), n,
                                            ptr(out), nthreads or os.cpu_count() or 1)
    if st != 0:
        raise ValueError(f"oracle decompress failed ({st})")
    return out


def chunk_trace(model: OracleModel, tokens: np.ndarray) -> dict:
    tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
    n = len(tokens)
    V, d, nl = model.vocab, model.d_model, model.n_layers
    logits = np.zeros((n, V), dtype=np.int32)
    lohi = np.zeros((n, 2), dtype=np.uint32)
    attn = np.zeros((n, nl, d), dtype=np.int8)
    fin = np.zeros((n, d), dtype=np.int8)
    lib().czo_chunk_trace(model.ref, ptr(tokens), n, ptr(logits), ptr(lohi), ptr(attn), ptr(fin))
    return {"logits": logits, "lohi": lohi, "attn": attn, "final_in": fin}


def build_cumfreqs(logits: np.ndarray, lut: np.ndarray, coef: int, total: int) -> np.ndarray:
    lg = np.ascontiguousarray(logits, dtype=np.int32)
    lut = np.ascontiguousarray(lut, dtype=np.uint16)
    cum = np.zeros(len(lg), dtype=np.uint32)
    lib().czo_build_cumfreqs(ptr(lg), len(lg), ptr(lut), coef, total, ptr(cum))
    return cum


def encode_symbols(cum_rows, symbols) -> bytes:
    """Arithmetic-encode symbols, row i of cum_rows being the CDF of symbol i."""
    n = len(symbols)
    buf = np.zeros(slot_cap(max(n, 1)), dtype=np.uint8)
    e = Encoder()
    L = lib()
    L.czo_enc_init(C.byref(e), ptr(buf), len(buf))
    for row, s in zip(cum_rows, symbols):
        row = np.ascontiguousarray(row, dtype=np.uint32)
        L.czo_enc_encode(C.byref(e), ptr(row), len(row), int(s))
    L.czo_enc_finish(C.byref(e))
    assert not e.overflow
    return buf[: e.len].tobytes()


def encode_intervals(pairs, total: int) -> bytes:
    """Arithmetic-encode (sym_low, sym_high) pairs directly (arith_coder.rs:80-130)."""
    n = len(pairs)
    buf = np.zeros(slot_cap(max(n, 1)), dtype=np.uint8)
    e = Encoder()
    L = lib()
    L.czo_enc_init(C.byref(e), ptr(buf), len(buf))
    for lo, hi in pairs:
        L.czo_enc_encode_range(C.byref(e), int(lo), int(hi), int(total))
    L.czo_enc_finish(C.byref(e))
    assert not e.overflow
    return buf[: e.len].tobytes()


def decode_symbols(data: bytes, cum_rows) -> list[int]:
    arr = np.frombuffer(data + b"\0", dtype=np.uint8).copy()
    d = Decoder()
    L = lib()
    L.czo_dec_init(C.byref(d), ptr(arr), len(data))
    out = []
    for row in cum_rows:
        row = np.ascontiguousarray(row, dtype=np.uint32)
        out.append(L.czo_dec_decode(C.byref(d), ptr(row), len(row)))
    return out


def attention_seq(q: np.ndarray, k: np.ndarray, v: np.ndarray, score_mult, cos, sin, lut,
                  sink_key=None) -> np.ndarray:
    """q: [n][H][64], k/v: [n][64] (k, q before RoPE) -> out [n][H][64]."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    k = np.ascontiguousarray(k, dtype=np.int8)
    v = np.ascontiguousarray(v, dtype=np.int8)
    n, H = q.shape[0], q.shape[1]
    sm = np.ascontiguousarray(score_mult, dtype=np.int32)
    cos = np.ascontiguousarray(cos, dtype=np.int16)
    sin = np.ascontiguousarray(sin, dtype=np.int16)
    lut = np.ascontiguousarray(lut, dtype=np.uint16)
    sk = None if sink_key is None else np.ascontiguousarray(sink_key, dtype=np.int8)
    out = np.zeros((n, H, 64), dtype=np.int8)
    lib().czo_attention_seq(ptr(q), ptr(k), ptr(v), n, H, ptr(sm), None if sk is None else ptr(sk),
                            ptr(cos), ptr(sin), ptr(lut), ptr(out))
    return out
