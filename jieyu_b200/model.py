"""Host-side mirror of the reference's model objects, backed by libjieyu_b200.

* ``Config``      — hyper-parameters (the reference's ModelInfo / ModelRefs fields).
* ``HostWeights`` — host buffers in the reference's own layouts (Q8_0 blocks
  [out][in/32]x34 B, fp32 or fp16 [in][out], fp32 norms/biases) plus the
  ``LayerWeights`` / ``jyc_model_desc`` structs that point at them, i.e. what
  ``bind_model`` produces (libs/model_libs/pipeline.h:63-153).
* ``DeviceModel`` — the uploaded model: ``generate`` mirrors ``generate()``
  (libs/model_libs/generate.h:90-112) and runs entirely on the GPU.

Synthetic weights are a pure integer function of (seed, stream, index)
(``jyc_synth_*``), so every process — and the CPU checker — sees the same bytes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace
from typing import Callable, Optional

import numpy as np

from . import _capi
from ._capi import JYC_Q8_0, LayerWeights, ModelDesc, WMat, check


@dataclass(frozen=True)
class Config:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    theta: float
    wtype: str = "q8"          # linear weights: "q8" (Q8_0), "f32", "f16" or "kq" (Q4_K / Q5_K / Q6_K blocks)
    embed: str = "f32"         # "f32", "f16", "q8" (separate) or "tied" (Q8_0, = LM head)
    qkv_bias: bool = False
    max_seq: int = 512
    prompt_len: int = 32
    new_tokens: int = 128
    std: float = 0.02
    embed_rows: int = 0        # embedding rows when the LM head holds a vocabulary slice (0: vocab)
    vocab_offset: int = 0      # token id of the LM head's first row

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


# BASELINE.json configs (shapes as stated there).
CONFIGS = {
    # tiny Llama-style, Q8_0 linears, fp32 embedding/norms, max context 512
    "c0": Config("c0_tiny", 512, 8, 8, 4, 64, 1376, 32000, 1e4, "q8", "f32", False, 512, 32, 128),
    # Qwen2.5-0.5B shape, tied Q8_0 embedding, QKV bias, theta 1e6
    "c1": Config("c1_qwen2.5_0.5b", 896, 24, 14, 2, 64, 4864, 151936, 1e6, "q8", "tied", True,
                 1024, 512, 256),
    # Llama-3.2-1B shape (Q8_0 and fp32 variants)
    # max_seq covers the longest decode context it is measured at (16384) + steps
    "c2": Config("c2_llama3.2_1b", 2048, 16, 32, 8, 64, 8192, 128256, 5e5, "q8", "q8", False,
                 16512, 2048, 128),
    "c2f": Config("c2_llama3.2_1b_f32", 2048, 16, 32, 8, 64, 8192, 128256, 5e5, "f32", "f32",
                  False, 16512, 2048, 128),
    # Llama-3-8B shape
    "c3": Config("c3_llama3_8b", 4096, 32, 32, 8, 128, 14336, 128256, 5e5, "q8", "q8", False,
                 4352, 4096, 128),
    # batched decode sweep on the Llama-3.2-1B shape (Q8_0), every
    # sequence at context 2048 + 128 greedy tokens
    "c4": Config("c4_llama3.2_1b_batched", 2048, 16, 32, 8, 64, 8192, 128256, 5e5, "q8", "q8", False,
                 2304, 2048, 128),
}

# Stream ids of the synthetic generator (one per tensor).
_SLOTS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6, "bq": 7, "bk": 8, "bv": 9}
STREAM_EMBED = 1 << 20
STREAM_HEAD = (1 << 20) + 1
STREAM_PROMPT = 1 << 21


def _stream(layer: int, slot: str) -> int:
    return layer * 16 + _SLOTS[slot]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def synth_q8(seed: int, stream: int, rows: int, k: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(rows * (k // 32) * 34, dtype=np.uint8)
    check(_capi.load().jyc_synth_q8_0(seed, stream, std, _ptr(out), rows, k))
    return out


def synth_f32(seed: int, stream: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    check(_capi.load().jyc_synth_f32(seed, stream, std, _ptr(out), n))
    return out


def synth_ids(seed: int, stream: int, vocab: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    check(_capi.load().jyc_synth_ids(seed, stream, vocab, _ptr(out), n))
    return out


def quantize_q8(x: np.ndarray, rows: int, k: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(rows * (k // 32) * 34, dtype=np.uint8)
    check(_capi.load().jyc_quantize_q8_0(_ptr(x), _ptr(out), rows, k))
    return out


def rope_table(max_seq: int, head_dim: int, theta: float):
    """cos/sin tables exactly as RoPETable::init (libs/date_libs/date.h:52-66)."""
    half = head_dim // 2
    c = np.empty(max_seq * half, dtype=np.float32)
    s = np.empty(max_seq * half, dtype=np.float32)
    check(_capi.load().jyc_rope_table(max_seq, head_dim, theta, _ptr(c), _ptr(s)))
    return c, s


def prompt_ids(cfg: Config, seed: int = 1234, index: int = 0, n: Optional[int] = None) -> np.ndarray:
    """Uniform-random prompt ids in [0, vocab) (seeded)."""
    return synth_ids(seed, STREAM_PROMPT + index, cfg.vocab, cfg.prompt_len if n is None else n)


class HostWeights:
    """Host tensors in the reference layouts + the descriptor pointing at them."""

    def __init__(self, cfg: Config, tensors: dict, cos: np.ndarray, sin: np.ndarray, qtypes: Optional[dict] = None):
        self.cfg = cfg
        self.t = tensors          # keeps every buffer alive
        self.qt = dict(qtypes or {})  # block type (JYC_Q4K / Q5K / Q6K) of uint8 tensors; Q8_0 when absent
        self.cos, self.sin = cos, sin
        self._build_desc()

    # -- constructors -------------------------------------------------------
    @classmethod
    def synthetic(cls, cfg: Config, seed: int = 1234) -> "HostWeights":
        D, F, L = cfg.hidden, cfg.inter, cfg.layers
        t: dict = {}
        ones = np.ones(D, dtype=np.float32)
        for l in range(L):
            t[f"rms1.{l}"] = ones
            t[f"rms2.{l}"] = ones
            shapes = {"q": (cfg.q_dim, D), "k": (cfg.kv_dim, D), "v": (cfg.kv_dim, D),
                      "o": (D, cfg.q_dim), "gate": (F, D), "up": (F, D), "down": (D, F)}
            for name, (out, inn) in shapes.items():
                if cfg.wtype == "q8":
                    t[f"{name}.{l}"] = synth_q8(seed, _stream(l, name), out, inn, cfg.std)
                else:  # fp32 [in][out]
                    t[f"{name}.{l}"] = synth_f32(seed, _stream(l, name), inn * out, cfg.std)
            if cfg.qkv_bias:
                t[f"bq.{l}"] = synth_f32(seed, _stream(l, "bq"), cfg.q_dim, cfg.std)
                t[f"bk.{l}"] = synth_f32(seed, _stream(l, "bk"), cfg.kv_dim, cfg.std)
                t[f"bv.{l}"] = synth_f32(seed, _stream(l, "bv"), cfg.kv_dim, cfg.std)
        V = cfg.vocab
        if cfg.embed == "tied":
            t["head"] = synth_q8(seed, STREAM_HEAD, V, D, cfg.std)
        else:
            if cfg.wtype == "q8":
                t["head"] = synth_q8(seed, STREAM_HEAD, V, D, cfg.std)
            else:
                t["head"] = synth_f32(seed, STREAM_HEAD, D * V, cfg.std)  # [hidden][vocab]
            if cfg.embed == "q8":
                t["embed"] = synth_q8(seed, STREAM_EMBED, V, D, cfg.std)
            else:
                t["embed"] = synth_f32(seed, STREAM_EMBED, V * D, cfg.std)
        t["final_norm"] = ones
        cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
        return cls(cfg, t, cos, sin)

    @classmethod
    def synthetic_f16(cls, cfg: Config, seed: int = 1234) -> "HostWeights":
        """The seeded fp32 weights of `synthetic` (fp32 variant of cfg), every
        linear matrix, the LM head and the embedding rounded to fp16 (IEEE
        halves, round to nearest even) in the reference's [in][out] layout."""
        f = cls.synthetic(replace(cfg, wtype="f32", embed="f32"), seed)
        t = {}
        for key, a in f.t.items():
            two_d = key.split(".")[0] in ("q", "k", "v", "o", "gate", "up", "down", "head", "embed")
            t[key] = a.astype(np.float16).view(np.uint16) if two_d else a
        return cls(replace(cfg, wtype="f16", embed="f16"), t, f.cos, f.sin)

    @classmethod
    def synthetic_kquant(cls, cfg: Config, seed: int = 1234) -> "HostWeights":
        """Seeded K-quant weights (the formats of the reference's downloads),
        mixed per matrix as Q4_K_M files mix them: Q, O, gate Q4_K; K, up
        Q5_K; V, down, the LM head and the embedding Q6_K. Random quant bytes;
        the fp16 block scales drawn so that weights stay O(0.01-0.1); unit
        norms. Needs hidden, heads*head_dim and intermediate multiples of 256."""
        D, F, V, qd, kvd = cfg.hidden, cfg.inter, cfg.vocab, cfg.q_dim, cfg.kv_dim
        bb = {0: 144, 1: 176, 2: 210}
        rng = np.random.default_rng(seed)
        stream = [seed * 0x9E3779B9 & 0xFFFFFFFF]

        def hash_bytes(nbytes: int) -> np.ndarray:
            # counter-based bytes (the lowbias32 integer mix), fast for GBs
            x = np.arange(stream[0], stream[0] + (nbytes + 3) // 4, dtype=np.uint64).astype(np.uint32)
            stream[0] = (stream[0] + (nbytes + 3) // 4) & 0xFFFFFFFF
            x ^= x >> np.uint32(16)
            x *= np.uint32(0x7FEB352D)
            x ^= x >> np.uint32(15)
            x *= np.uint32(0x846CA68B)
            x ^= x >> np.uint32(16)
            return x.view(np.uint8)[:nbytes]

        def blocks(q: int, n: int, k: int, lo: float, hi: float) -> np.ndarray:
            nb = n * (k // 256)
            b = hash_bytes(nb * bb[q]).reshape(nb, bb[q]).copy()
            d = rng.uniform(lo, hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
            if q == 2:
                b[:, 208:210] = d
            else:
                b[:, 0:2] = d
                b[:, 2:4] = rng.uniform(lo, hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
            return np.ascontiguousarray(b.reshape(-1))

        kinds = {"q": 0, "k": 1, "v": 2, "o": 0, "gate": 0, "up": 1, "down": 2}
        dims = {"q": (qd, D), "k": (kvd, D), "v": (kvd, D), "o": (D, qd), "gate": (F, D), "up": (F, D),
                "down": (D, F)}
        t, qt = {}, {}
        ones = np.ones(D, dtype=np.float32)
        for l in range(cfg.layers):
            t[f"rms1.{l}"] = ones
            t[f"rms2.{l}"] = ones
            for key, q in kinds.items():
                lo, hi = (2.0 ** -17, 2.0 ** -15) if q == 2 else (2.0 ** -13, 2.0 ** -11)
                t[f"{key}.{l}"] = blocks(q, *dims[key], lo, hi)
                qt[f"{key}.{l}"] = q
        t["head"] = blocks(2, V, D, 2.0 ** -15, 2.0 ** -13)
        t["embed"] = blocks(2, V, D, 2.0 ** -12, 2.0 ** -10)
        qt["head"] = qt["embed"] = 2
        t["final_norm"] = ones
        cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
        return cls(replace(cfg, wtype="kq", embed="q8", qkv_bias=False), t, cos, sin, qtypes=qt)

    @classmethod
    def bind_test_kat(cls) -> "HostWeights":
        """The fp32 model of the reference's check_bind_weights
        (libs/text/text.h:485-541 gen_weights::build with make_weights' lm_head,
        text.h:604-610): pseudo(i) = ((i*37)%19-9)/8, RoPE from bind_model's
        RoPETable::init with theta 10000."""
        cfg = Config("kat_bind", 8, 2, 2, 1, 4, 16, 24, 10000.0, "f32", "f32", False, 8, 3, 3)

        def pseudo(n: int, off: int, mul: float) -> np.ndarray:
            i = np.arange(n, dtype=np.int64) + off
            return (((i * 37) % 19 - 9).astype(np.float32) / np.float32(8.0)) * np.float32(mul)

        D, qd, kvd, F, V = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter, cfg.vocab
        t = {}
        for l in range(cfg.layers):
            t[f"rms1.{l}"] = np.float32(1.0) + pseudo(D, 3 * l, 0.25)
            t[f"rms2.{l}"] = np.float32(1.0) + pseudo(D, 5 * l, 0.25)
            t[f"q.{l}"] = pseudo(D * qd, 7 * l, 0.5)
            t[f"k.{l}"] = pseudo(D * kvd, 11 * l, 0.5)
            t[f"v.{l}"] = pseudo(D * kvd, 13 * l, 0.5)
            t[f"o.{l}"] = pseudo(qd * D, 17 * l, 0.5)
            t[f"gate.{l}"] = pseudo(D * F, 19 * l, 0.5)
            t[f"down.{l}"] = pseudo(F * D, 23 * l, 0.5)
            t[f"up.{l}"] = pseudo(D * F, 29 * l, 0.5)
        t["embed"] = pseudo(V * D, 101, 0.5)
        t["head"] = pseudo(D * V, 211, 2.0)
        t["final_norm"] = np.float32(1.0) + pseudo(D, 307, 0.25)
        cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
        return cls(cfg, t, cos, sin)

    @classmethod
    def shift_demo_kat(cls) -> "HostWeights":
        """The converter's demo model used by check_pipeline
        (libs/model_libs/converter.h:422-503): identity embedding for byte ids,
        zero attention/FFN, lm_head[v][v-1] = 1 (stored [in][out] after
        conversion), so greedy decoding emits id+1. max_seq = 1024 as the
        C ABI derives it from max_position_embeddings (main.hpp:64-67)."""
        cfg = Config("kat_shift", 256, 2, 8, 2, 32, 64, 259, 10000.0, "f32", "f32", False, 1024, 8, 16)
        D, qd, kvd, F, V = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.inter, cfg.vocab
        t = {}
        ones = np.ones(D, dtype=np.float32)
        for l in range(cfg.layers):
            t[f"rms1.{l}"] = ones
            t[f"rms2.{l}"] = ones
            for name, n in (("q", D * qd), ("k", D * kvd), ("v", D * kvd), ("o", qd * D),
                            ("gate", D * F), ("up", D * F), ("down", F * D)):
                t[f"{name}.{l}"] = np.zeros(n, dtype=np.float32)
        emb = np.zeros((V, D), dtype=np.float32)
        for v in range(256):
            emb[v, v] = 1.0
        head = np.zeros((D, V), dtype=np.float32)  # [in][out]
        for v in range(1, 256):
            head[v - 1, v] = 1.0
        t["embed"] = emb.reshape(-1)
        t["head"] = head.reshape(-1)
        t["final_norm"] = ones
        cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
        return cls(cfg, t, cos, sin)

    # -- descriptor ---------------------------------------------------------
    def _wmat(self, key: str) -> WMat:
        a = self.t[key]
        if a.dtype == np.uint8:
            return WMat(None, None, _ptr(a), self.qt.get(key, JYC_Q8_0))
        if a.dtype == np.uint16:  # IEEE halves, [in][out] (matmul_f16.h)
            return WMat(None, _ptr(a), None, 0)
        return WMat(_ptr(a), None, None, 0)

    def _build_desc(self) -> None:
        cfg = self.cfg
        L = cfg.layers
        self.layer_arr = (LayerWeights * L)()
        for l in range(L):
            lw = self.layer_arr[l]
            lw.rms1_weight = _ptr(self.t[f"rms1.{l}"])
            lw.rms2_weight = _ptr(self.t[f"rms2.{l}"])
            lw.Wq, lw.Wk, lw.Wv, lw.Wo = (self._wmat(f"{n}.{l}") for n in ("q", "k", "v", "o"))
            lw.W1, lw.W2, lw.W3 = (self._wmat(f"{n}.{l}") for n in ("gate", "down", "up"))
            for b in ("bq", "bk", "bv"):
                setattr(lw, b, _ptr(self.t[f"{b}.{l}"]) if f"{b}.{l}" in self.t else None)
        d = ModelDesc()
        d.layers = self.layer_arr
        d.num_layers = L
        d.lm_head = self._wmat("head")
        d.embed = self._wmat("head") if cfg.embed == "tied" else self._wmat("embed")
        d.final_rms_weight = _ptr(self.t["final_norm"])
        d.cos_table = _ptr(self.cos)
        d.sin_table = _ptr(self.sin)
        d.max_seq = cfg.max_seq
        d.vocab_size = cfg.vocab
        d.hidden = cfg.hidden
        d.num_heads = cfg.heads
        d.num_kv_heads = cfg.kv_heads
        d.head_dim = cfg.head_dim
        d.intermediate = cfg.inter
        d.embed_rows = cfg.embed_rows
        d.vocab_offset = cfg.vocab_offset
        self.desc = d

    def weight_bytes_per_token(self) -> float:
        """Algorithmic weight bytes one decode token reads (Q8_0: 34 B / 32)."""
        cfg = self.cfg
        D, F = cfg.hidden, cfg.inter
        per = {"q8": 34.0 / 32.0, "f16": 2.0}.get(cfg.wtype, 4.0)
        lin = (cfg.q_dim + 2 * cfg.kv_dim) * D + D * cfg.q_dim + 3 * F * D
        b = cfg.layers * (lin * per + 2 * D * 4 + (cfg.q_dim + 2 * cfg.kv_dim) * 4 * cfg.qkv_bias)
        names = ("q", "k", "v", "o", "gate", "up", "down")
        if cfg.wtype == "kq" and all(f"{n}.{l}" in self.qt for l in range(cfg.layers) for n in names):
            # every layer matrix K-quant: the device reads the blocks in place
            b -= cfg.layers * lin * per
            b += sum(self.t[f"{n}.{l}"].nbytes for l in range(cfg.layers) for n in names)
        head_q8 = self.t["head"].dtype == np.uint8 and self.qt.get("head", JYC_Q8_0) == JYC_Q8_0
        head_b = 34.0 / 32.0 if head_q8 else 2.0 if self.t["head"].dtype == np.uint16 else 4.0
        b += cfg.vocab * D * head_b + 4 * D
        emb_key = "head" if cfg.embed == "tied" else "embed"
        emb_q8 = self.t[emb_key].dtype == np.uint8 and self.qt.get(emb_key, JYC_Q8_0) == JYC_Q8_0
        b += D * (34.0 / 32.0 if emb_q8 else 4.0)
        return b


class DeviceModel:
    """A model resident in HBM (jyc_model_create uploads once)."""

    def __init__(self, hw: HostWeights):
        self.hw = hw
        self.cfg = hw.cfg
        self.lib = _capi.load()
        h = self.lib.jyc_model_create(C.byref(hw.desc))
        if not h:
            raise _capi.JycError(-1, _capi.last_error())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.jyc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate(self, prompt: np.ndarray, max_new: int, eos: Optional[list] = None,
                 temperature: float = 0.0, repetition_penalty: float = 1.0,
                 cb: Optional[Callable[[int], bool]] = None) -> np.ndarray:
        """generate() contract: returns out_ids[:len] (prompt + new tokens)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(self.cfg.max_seq + 1, dtype=np.int32)
        e = np.ascontiguousarray(eos if eos else [0], dtype=np.int32)
        ccb = _capi.TOKEN_CB(lambda i, ud: 1 if cb(i) else 0) if cb else _capi.TOKEN_CB()
        n = check(self.lib.jyc_generate(self.h, _ptr(prompt), len(prompt), _ptr(e),
                                        len(eos) if eos else 0, max_new, temperature, _ptr(out),
                                        repetition_penalty, ccb, None))
        return out[:n].copy()

    def forward_logits(self, ids: np.ndarray, start_pos: int, want_hidden: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        hid = np.empty(self.cfg.hidden, dtype=np.float32) if want_hidden else None
        check(self.lib.jyc_forward_logits(self.h, _ptr(ids), len(ids), start_pos, _ptr(logits),
                                          _ptr(hid) if hid is not None else None))
        return (logits, hid) if want_hidden else logits

    def read_kv(self, layer: int, npos: int):
        cfg = self.cfg
        k = np.empty(npos * cfg.kv_dim, dtype=np.int8)
        v = np.empty_like(k)
        ks = np.empty(npos * cfg.kv_heads, dtype=np.float32)
        vs = np.empty_like(ks)
        check(self.lib.jyc_model_read_kv(self.h, layer, npos, _ptr(k), _ptr(ks), _ptr(v), _ptr(vs)))
        return k, ks, v, vs

    def write_kv(self, layer: int, k: np.ndarray, ks: np.ndarray, v: np.ndarray, vs: np.ndarray) -> None:
        """Positions [0, npos) of one layer's cache from host arrays in the
        reference's __KVcache order (k, v int8 [npos][kv][hd]; ks, vs fp32 [npos][kv])."""
        cfg = self.cfg
        npos = len(ks) // cfg.kv_heads
        k, v = (np.ascontiguousarray(a, dtype=np.int8) for a in (k, v))
        ks, vs = (np.ascontiguousarray(a, dtype=np.float32) for a in (ks, vs))
        assert k.size == npos * cfg.kv_dim and v.size == k.size and vs.size == ks.size
        check(self.lib.jyc_model_write_kv(self.h, layer, npos, _ptr(k), _ptr(ks), _ptr(v), _ptr(vs)))

    # device-resident stepping (bench)
    def prefill_device(self, ids_dev_ptr: int, n: int, stream: int) -> None:
        check(self.lib.jyc_prefill_device(self.h, ids_dev_ptr, n, stream))

    def decode_device(self, n_steps: int, stream: int) -> None:
        check(self.lib.jyc_decode_device(self.h, n_steps, stream))

    def rewind(self, length: int, stream: int) -> None:
        check(self.lib.jyc_model_rewind(self.h, length, stream))

    def length(self, stream: int) -> int:
        return check(self.lib.jyc_model_length(self.h, stream))

    def tokens_device_ptr(self) -> int:
        return self.lib.jyc_model_tokens_device(self.h)

    def kernels_per_step(self) -> int:
        return self.lib.jyc_model_kernels_per_step(self.h)


class BatchDecoder:
    """B independent sequences decoded together on one DeviceModel
    (jyc_batch_*): per-sequence prefill, then batched greedy steps."""

    def __init__(self, model: "DeviceModel", num_seqs: int):
        self.model = model
        self.lib = model.lib
        self.n = num_seqs
        h = self.lib.jyc_batch_create(model.h, num_seqs)
        if not h:
            raise _capi.JycError(-1, _capi.last_error())
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.jyc_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, seq: int, prompt: np.ndarray) -> None:
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        check(self.lib.jyc_batch_prefill(self.h, seq, _ptr(prompt), len(prompt)))

    def decode(self, n_steps: int, stream: int = 0) -> None:
        check(self.lib.jyc_batch_decode(self.h, n_steps, stream))

    def rewind(self, length: int, stream: int = 0) -> None:
        check(self.lib.jyc_batch_rewind(self.h, length, stream))

    def tokens(self, seq: int) -> np.ndarray:
        out = np.zeros(self.model.cfg.max_seq + 1, dtype=np.int32)
        n = check(self.lib.jyc_batch_tokens(self.h, seq, _ptr(out), len(out)))
        return out[:n].copy()

    def path(self) -> int:
        return self.lib.jyc_batch_path(self.h)

    def kernels_per_step(self) -> int:
        return self.lib.jyc_batch_kernels_per_step(self.h)


def with_max_seq(cfg: Config, max_seq: int) -> Config:
    return replace(cfg, max_seq=max_seq)
