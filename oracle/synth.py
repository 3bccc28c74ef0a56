"""TEST INFRASTRUCTURE ONLY — seeded synthetic models for the CPU checkers and
the reference arm of bench.py, built without the product library.

The weights are the counter-based generator of liboracle.so (jyo_synth_*,
byte-identical to the library's jyc_synth_*; a host test holds the two
equal), laid out as the reference's own structures expect: Q8_0 blocks
[out][in/32] x 34 B, fp32 norms of 1.0, RoPE tables from RoPETable::init
(jyo_rope_table, libs/date_libs/date.h:52-66). The ctypes structures mirror
jyc_wmat / jyc_layer_weights / jyc_model_desc of include/jieyu_b200.h, whose
layouts equal the reference's WMat / LayerWeights (oracle/ref_harness.cpp
static_asserts them against the reference headers).

Only the Q8_0 model shapes the bench times are needed here (tied or separate
embedding, optional QKV bias); the stream ids per tensor follow the
library's HostWeights.synthetic so both sides see the same bytes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from .bind import Oracle


class WMat(C.Structure):
    _fields_ = [("f", C.c_void_p), ("h", C.c_void_p), ("q", C.c_void_p), ("qt", C.c_uint8)]


class LayerWeights(C.Structure):
    _fields_ = [
        ("rms1_weight", C.c_void_p),
        ("Wq", WMat), ("Wk", WMat), ("Wv", WMat), ("Wo", WMat),
        ("bq", C.c_void_p), ("bk", C.c_void_p), ("bv", C.c_void_p),
        ("rms2_weight", C.c_void_p),
        ("W1", WMat), ("W2", WMat), ("W3", WMat),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("layers", C.POINTER(LayerWeights)), ("num_layers", C.c_int),
        ("embed", WMat), ("lm_head", WMat),
        ("final_rms_weight", C.c_void_p), ("cos_table", C.c_void_p), ("sin_table", C.c_void_p),
        ("max_seq", C.c_int), ("vocab_size", C.c_int), ("hidden", C.c_int), ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int), ("head_dim", C.c_int), ("intermediate", C.c_int),
        ("embed_rows", C.c_int), ("vocab_offset", C.c_int),
    ]


Q8_0 = 3
STREAM_EMBED = 1 << 20
STREAM_HEAD = (1 << 20) + 1
STREAM_PROMPT = 1 << 21
_SLOTS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "bq": 7, "bk": 8, "bv": 9}


@dataclass(frozen=True)
class Shape:
    """A Q8_0 model shape."""
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    theta: float
    embed: str = "q8"       # "q8" (separate Q8_0 embedding) or "tied" (= LM head)
    qkv_bias: bool = False
    std: float = 0.02


SHAPES = {
    "c1": Shape("c1_qwen2.5_0.5b", 896, 24, 14, 2, 64, 4864, 151936, 1e6, "tied", True),
    "c2": Shape("c2_llama3.2_1b", 2048, 16, 32, 8, 64, 8192, 128256, 5e5),
    "c3": Shape("c3_llama3_8b", 4096, 32, 32, 8, 128, 14336, 128256, 5e5),
}


class SynthModel:
    """Host weights of a seeded Q8_0 model and the descriptor pointing at them."""

    def __init__(self, shape: Shape, max_seq: int, seed: int = 1234, oracle: Oracle | None = None):
        o = oracle or Oracle()
        lib = o.lib
        lib.jyo_synth_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_size_t]
        lib.jyo_synth_q8_0.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_size_t, C.c_size_t]
        self.shape, self.max_seq, self.seed = shape, max_seq, seed
        s = shape
        D, F, qd, kvd = s.hidden, s.inter, s.heads * s.head_dim, s.kv_heads * s.head_dim
        self.t: dict = {}

        def q8(stream: int, rows: int, k: int) -> np.ndarray:
            out = np.empty(rows * (k // 32) * 34, np.uint8)
            lib.jyo_synth_q8_0(seed, stream, s.std, out.ctypes.data, rows, k)
            return out

        def f32(stream: int, n: int) -> np.ndarray:
            out = np.empty(n, np.float32)
            lib.jyo_synth_f32(seed, stream, s.std, out.ctypes.data, n)
            return out

        ones = np.ones(D, np.float32)
        self.t["ones"] = ones
        L = s.layers
        self.layer_arr = (LayerWeights * L)()
        shapes = {"q": (qd, D), "k": (kvd, D), "v": (kvd, D), "o": (D, qd), "gate": (F, D), "up": (F, D),
                  "down": (D, F)}
        for l in range(L):
            lw = self.layer_arr[l]
            lw.rms1_weight = lw.rms2_weight = ones.ctypes.data
            for name, (n, k) in shapes.items():
                a = self.t[f"{name}.{l}"] = q8(l * 16 + _SLOTS[name], n, k)
                setattr(lw, {"q": "Wq", "k": "Wk", "v": "Wv", "o": "Wo", "gate": "W1", "down": "W2",
                             "up": "W3"}[name], WMat(None, None, a.ctypes.data, Q8_0))
            if s.qkv_bias:
                for b, n in (("bq", qd), ("bk", kvd), ("bv", kvd)):
                    a = self.t[f"{b}.{l}"] = f32(l * 16 + _SLOTS[b], n)
                    setattr(lw, b, a.ctypes.data)
        head = self.t["head"] = q8(STREAM_HEAD, s.vocab, D)
        emb = head if s.embed == "tied" else q8(STREAM_EMBED, s.vocab, D)
        self.t["embed"] = emb
        half = s.head_dim // 2
        self.cos = np.empty(max_seq * half, np.float32)
        self.sin = np.empty(max_seq * half, np.float32)
        lib.jyo_rope_table(max_seq, s.head_dim, s.theta, self.cos.ctypes.data, self.sin.ctypes.data)
        d = ModelDesc()
        d.layers = self.layer_arr
        d.num_layers = L
        d.embed = WMat(None, None, emb.ctypes.data, Q8_0)
        d.lm_head = WMat(None, None, head.ctypes.data, Q8_0)
        d.final_rms_weight = ones.ctypes.data
        d.cos_table, d.sin_table = self.cos.ctypes.data, self.sin.ctypes.data
        d.max_seq, d.vocab_size, d.hidden = max_seq, s.vocab, D
        d.num_heads, d.num_kv_heads, d.head_dim, d.intermediate = s.heads, s.kv_heads, s.head_dim, F
        self.desc = d

    def weight_bytes_per_token(self) -> float:
        """Q8_0 bytes one decode token reads (layers + LM head + one embedding row)."""
        s = self.shape
        D, F, qd, kvd = s.hidden, s.inter, s.heads * s.head_dim, s.kv_heads * s.head_dim
        lin = (qd + 2 * kvd) * D + D * qd + 3 * F * D
        return s.layers * (lin * 34 / 32 + 2 * D * 4 + (qd + 2 * kvd) * 4 * s.qkv_bias) + s.vocab * D * 34 / 32 \
            + 4 * D + D * 34 / 32


def prompt(oracle: Oracle, vocab: int, n: int, seed: int = 1234, index: int = 0) -> np.ndarray:
    """Uniform-random ids in [0, vocab) (the library's prompt_ids stream)."""
    lib = oracle.lib
    lib.jyo_synth_ids.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_void_p, C.c_size_t]
    out = np.empty(n, np.int32)
    lib.jyo_synth_ids(seed, STREAM_PROMPT + index, vocab, out.ctypes.data, n)
    return out


def context_kv(layers: int, npos: int, kv_heads: int, head_dim: int, seed: int = 99):
    """Per layer: a seeded context of npos positions in the cache layout of
    __KVq ([pos][kv head][hd] int8 K and V, [pos][kv head] fp32 scales):
    int8 values in [-127, 127] and scales of 0.02-0.05 / 127-sized steps, the
    range kv_pack_q8 writes for activations of this model's size. Yields
    (layer, k, ks, v, vs)."""
    rng = np.random.default_rng(seed)
    for l in range(layers):
        k = rng.integers(-127, 128, size=npos * kv_heads * head_dim, dtype=np.int8)
        v = rng.integers(-127, 128, size=npos * kv_heads * head_dim, dtype=np.int8)
        ks = rng.uniform(0.2, 0.5, size=npos * kv_heads).astype(np.float32) / np.float32(127.0)
        vs = rng.uniform(0.02, 0.05, size=npos * kv_heads).astype(np.float32) / np.float32(127.0)
        yield l, k, ks, v, vs
