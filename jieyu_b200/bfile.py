"""Model directories in the reference's runtime format: `model.bf` (tensor
file, version 2 with a tensor directory) + `model_info.json`.

The reference converts checkpoints (safetensors, GGUF) into this format once
(libs/model_libs/converter.h, libs/gguf_libs/gguf_convert.h:201-229 copies
Q8_0 blocks verbatim) and its runtime maps the file and binds tensors by
name (libs/model_libs/bfile.h:141-204 View::open, load_weights.h:97-155
bind_layers / bind_biases / bind_embed / bind_lm_head / bind_final_norm,
pipeline.h:63-153 bind_model's shape checks). `load_model_dir` does the same
on the host: the file is memory-mapped, every weight is a zero-copy view of
its bytes, and the result is a `HostWeights` whose descriptor the device
path uploads (`DeviceModel`). `write_bfile` writes byte-identical files to
the reference's writer (bfile.h:275-343), which the tests check.

File layout (all integers little-endian):
  header, 64 bytes: "JYAIBF", hidden u64 @6, layers u64 @14, mode u8 @22,
    num_heads u8 @23, num_kv_heads u8 @24, head_dim u8 @25,
    intermediate u32 @26, vocab u64 @30, version u32 @38 (2),
    tensor count u32 @42, data offset u32 @46, entry size u32 @50 (104)
  directory: count x 104-byte entries {name char[64], dtype u8, ndim u8,
    u16, shape u32[4], u32, offset u64 (from the data offset), nbytes u64}
  zero padding to the data offset (a multiple of 64), then each tensor's
    bytes at its offset (multiples of 64), zero padding between tensors.
Linear weights are stored [in][out] in f32 and [out][in/32] Q8_0 blocks.
"""
from __future__ import annotations

import json
import os
import numpy as np

from .model import Config, HostWeights, rope_table

MAGIC = b"JYAIBF"
VERSION = 2
HEADER = 64
ENTRY = 104
ALIGN = 64

F32, F16, BF16, I8, I32, Q4K, Q5K, Q6K, Q8_0 = range(9)
_ELEM = {F32: 4, I32: 4, F16: 2, BF16: 2, I8: 1}
_BLOCK = {Q4K: (256, 144), Q5K: (256, 176), Q6K: (256, 210), Q8_0: (32, 34)}
DTYPE_NAMES = {F32: "f32", F16: "f16", BF16: "bf16", I8: "i8", I32: "i32", Q4K: "q4_K", Q5K: "q5_K",
               Q6K: "q6_K", Q8_0: "q8_0"}

_ENTRY_DT = np.dtype([("name", "S64"), ("dtype", "u1"), ("ndim", "u1"), ("r0", "<u2"), ("shape", "<u4", (4,)),
                      ("r1", "<u4"), ("offset", "<u8"), ("nbytes", "<u8")])
assert _ENTRY_DT.itemsize == ENTRY

# bfile dtype codes of the K-quants <-> the descriptor's JYC_Q4K / Q5K / Q6K
_KQ_CODE = {Q4K: 0, Q5K: 1, Q6K: 2}
_KQ_FILE = {v: k for k, v in _KQ_CODE.items()}

LAYER_SUFFIX = {  # load_weights.h:55-68, our tensor key -> reference name suffix
    "rms1": "input_layernorm.weight", "q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight",
    "v": "self_attn.v_proj.weight", "o": "self_attn.o_proj.weight", "rms2": "post_attention_layernorm.weight",
    "gate": "mlp.gate_proj.weight", "down": "mlp.down_proj.weight", "up": "mlp.up_proj.weight",
}
BIAS_SUFFIX = {"bq": "self_attn.q_proj.bias", "bk": "self_attn.k_proj.bias", "bv": "self_attn.v_proj.bias"}


class BFileError(ValueError):
    """A model.bf or model directory the reference's loader would reject."""


def tensor_bytes(dtype: int, elems: int) -> int:
    """Bytes of `elems` elements (0 for an unknown dtype or a partial block)."""
    if dtype in _BLOCK:
        be, bb = _BLOCK[dtype]
        return 0 if elems % be else elems // be * bb
    return elems * _ELEM.get(dtype, 0)


def _align(v: int) -> int:
    return (v + ALIGN - 1) // ALIGN * ALIGN


def layer_name(l: int, suffix: str) -> str:
    return f"model.layers.{l}.{suffix}"


class Tensor:
    """One directory entry with a zero-copy view of its bytes."""

    __slots__ = ("name", "dtype", "shape", "offset", "nbytes", "raw")

    def __init__(self, name, dtype, shape, offset, nbytes, raw):
        self.name, self.dtype, self.shape = name, dtype, tuple(shape)
        self.offset, self.nbytes, self.raw = offset, nbytes, raw

    def array(self) -> np.ndarray:
        """f32 / i32 / f16 / bf16 / i8 tensors as typed 1-D views; block
        formats as their raw bytes (uint8)."""
        if self.dtype == F32:
            return self.raw.view(np.float32)
        if self.dtype == I32:
            return self.raw.view(np.int32)
        if self.dtype in (F16, BF16):
            return self.raw.view(np.uint16)
        if self.dtype == I8:
            return self.raw.view(np.int8)
        return self.raw


class BFile:
    """A model.bf opened read-only (memory-mapped); validation follows the
    reference's View::open (bfile.h:141-176)."""

    def __init__(self, path: str):
        self.path = path
        size = os.path.getsize(path)
        if size < HEADER:
            raise BFileError(f"{path}: {size} bytes, shorter than the 64-byte header")
        self.map = np.memmap(path, dtype=np.uint8, mode="r")
        head = bytes(self.map[:HEADER])
        if head[:6] != MAGIC:
            raise BFileError(f"{path}: magic is {head[:6]!r}, not {MAGIC!r}")
        u32 = lambda o: int.from_bytes(head[o:o + 4], "little")  # noqa: E731
        u64 = lambda o: int.from_bytes(head[o:o + 8], "little")  # noqa: E731
        self.hidden, self.layers, self.mode = u64(6), u64(14), head[22]
        self.num_heads, self.num_kv_heads, self.head_dim = head[23], head[24], head[25]
        self.intermediate, self.vocab = u32(26), u64(30)
        self.version, count, self.data_off, esize = u32(38), u32(42), u32(46), u32(50)
        if self.version < VERSION:
            raise BFileError(f"{path}: version {self.version} has no tensor directory (needs {VERSION})")
        if esize != ENTRY:
            raise BFileError(f"{path}: directory entries of {esize} bytes, expected {ENTRY}")
        if self.data_off < HEADER or self.data_off > size:
            raise BFileError(f"{path}: data offset {self.data_off} outside the file")
        if HEADER + count * ENTRY > self.data_off:
            raise BFileError(f"{path}: {count} directory entries do not fit before the data offset")
        ents = np.frombuffer(self.map, dtype=_ENTRY_DT, count=count, offset=HEADER)
        self.tensors: dict[str, Tensor] = {}
        for e in ents:
            name = e["name"].split(b"\0", 1)[0].decode("utf-8", "replace")
            dt, nd = int(e["dtype"]), int(e["ndim"])
            if nd > 4:
                raise BFileError(f"{path}: {name}: {nd} dimensions (at most 4)")
            if tensor_bytes(dt, 1) == 0 and dt not in _BLOCK:
                raise BFileError(f"{path}: {name}: unknown dtype {dt}")
            shape = [int(s) for s in e["shape"][:nd]]
            elems = int(np.prod(shape, dtype=np.uint64)) if nd else 1
            off, nb = int(e["offset"]), int(e["nbytes"])
            if tensor_bytes(dt, elems) != nb:
                raise BFileError(f"{path}: {name}: shape {shape} of {DTYPE_NAMES[dt]} is not {nb} bytes")
            if off % ALIGN:
                raise BFileError(f"{path}: {name}: data offset {off} not a multiple of {ALIGN}")
            if self.data_off + off + nb > size:
                raise BFileError(f"{path}: {name}: data runs past the end of the file")
            if name not in self.tensors:  # the reference's find() takes the first match
                start = self.data_off + off
                self.tensors[name] = Tensor(name, dt, shape, start, nb, self.map[start:start + nb])

    def get(self, name: str) -> Tensor | None:
        return self.tensors.get(name)


def write_bfile(path: str, header: dict, tensors: list) -> None:
    """Writes a model.bf the way the reference's bfile::write_bfile does.
    header: hidden, layers, mode (default 1), num_heads, num_kv_heads,
    head_dim, intermediate, vocab. tensors: (name, dtype, shape, bytes)
    in file order."""
    dir_bytes = len(tensors) * ENTRY
    data_off = _align(HEADER + dir_bytes)
    offs, cur = [], 0
    for name, dt, shape, data in tensors:
        nb = len(memoryview(data).cast("B"))
        enc = name.encode()
        if not 1 <= len(enc) <= 63:
            raise BFileError(f"tensor name must be 1..63 bytes: {name}")
        if len(shape) > 4:
            raise BFileError(f"{name}: more than 4 dimensions")
        if tensor_bytes(dt, int(np.prod(shape, dtype=np.uint64)) if shape else 1) != nb:
            raise BFileError(f"{name}: shape {list(shape)} does not match {nb} bytes")
        offs.append(cur)
        cur = _align(cur + nb)
    head = bytearray(HEADER)
    head[0:6] = MAGIC
    head[6:14] = int(header["hidden"]).to_bytes(8, "little")
    head[14:22] = int(header["layers"]).to_bytes(8, "little")
    head[22] = int(header.get("mode", 1))
    head[23], head[24], head[25] = int(header["num_heads"]), int(header["num_kv_heads"]), int(header["head_dim"])
    head[26:30] = int(header["intermediate"]).to_bytes(4, "little")
    head[30:38] = int(header["vocab"]).to_bytes(8, "little")
    head[38:42] = VERSION.to_bytes(4, "little")
    head[42:46] = len(tensors).to_bytes(4, "little")
    head[46:50] = data_off.to_bytes(4, "little")
    head[50:54] = ENTRY.to_bytes(4, "little")
    ents = np.zeros(len(tensors), dtype=_ENTRY_DT)
    for i, (name, dt, shape, data) in enumerate(tensors):
        ents[i]["name"] = name.encode()
        ents[i]["dtype"], ents[i]["ndim"] = dt, len(shape)
        ents[i]["shape"][:len(shape)] = shape
        ents[i]["offset"], ents[i]["nbytes"] = offs[i], len(memoryview(data).cast("B"))
    with open(path, "wb") as f:
        f.write(head)
        f.write(ents.tobytes())
        f.write(b"\0" * (data_off - HEADER - dir_bytes))
        written = 0
        for (name, dt, shape, data), off in zip(tensors, offs):
            if off > written:
                f.write(b"\0" * (off - written))
            f.write(memoryview(data).cast("B"))
            written = off + len(memoryview(data).cast("B"))


def _first_pairs(pairs: list) -> dict:
    """An object's members with the first of duplicate keys kept, as the
    reference's json_file::find returns the first match."""
    out: dict = {}
    for k, v in pairs:
        out.setdefault(k, v)
    return out


def _read_info(path: str) -> dict:
    """model_info.json with numbers kept as their source text (the
    reference's parser keeps every value's raw text, json_parser.h:99)."""
    if not os.path.exists(path):
        raise BFileError(f"{path} not found")
    with open(path, encoding="utf-8") as f:
        return json.load(f, parse_int=str, parse_float=str, parse_constant=str, object_pairs_hook=_first_pairs)


def _info_text(info: dict, key: str) -> str:
    """json_file::GetJsonData (json.h:57-63): a string's text, else the
    value's source text; "" when the key is absent."""
    if key not in info:
        return ""
    v = info[key]
    if isinstance(v, str):
        return v
    if isinstance(v, bool):
        return "true" if v else "false"
    if v is None:
        return "null"
    return json.dumps(v, separators=(",", ":"))


def _info_int(info: dict, key: str, fallback: int) -> int:
    """json_file::GetJsonInt (json.h:73-83): std::stoi of the value's text
    (leading white space, a sign, then the digits it starts with), the
    fallback when the text is empty, has no digits or leaves the int range."""
    s = _info_text(info, key).lstrip(" \t\n\v\f\r")
    j = 1 if s[:1] in ("+", "-") else 0
    k = j
    while k < len(s) and s[k] in "0123456789":
        k += 1
    if k == j:
        return fallback
    v = int(s[:k])
    return v if -2 ** 31 <= v < 2 ** 31 else fallback


def load_model_dir(path: str, max_seq: int = 0, name: str | None = None) -> HostWeights:
    """Binds a reference model directory (model.bf + model_info.json) for the
    device path, with the reference's binding rules: per layer the nine
    tensors of load_weights.h:55-68 (norms f32; linear weights all Q8_0, all
    f16, all K-quant (Q4_K / Q5_K / Q6_K, read in place on the device), or a
    mix of f32 and the K-quants, which the device dequantises to fp32 once),
    optional q/k/v biases,
    model.embed_tokens.weight (f32, f16, Q8_0 or K-quant), lm_head.weight or
    (block formats only) the embedding as a tied head, model.norm.weight; shapes as bind_model checks
    them (pipeline.h:99-139). max_seq 0 takes max_position_embeddings
    clamped to [64, 4096], as the reference's C ABI does (main.hpp:64-67);
    RoPE theta is model_info's integer rope_theta (default 10000)."""
    bf = BFile(os.path.join(path, "model.bf"))
    info = _read_info(os.path.join(path, "model_info.json"))
    L, D, H, KV, hd = int(bf.layers), int(bf.hidden), int(bf.num_heads), int(bf.num_kv_heads), int(bf.head_dim)
    F, V = int(bf.intermediate), int(bf.vocab)
    if L <= 0 or D <= 0 or hd <= 0 or H <= 0:
        raise BFileError(f"{path}: header hyper-parameters are not valid (layers {L}, hidden {D}, heads {H})")
    qd, kvd = H * hd, KV * hd

    def need(key: str) -> Tensor:
        t = bf.get(key)
        if t is None:
            raise BFileError(f"{path}: missing tensor {key}")
        return t

    def expect(t: Tensor, shape: tuple) -> None:
        if t.shape != tuple(shape):
            raise BFileError(f"{path}: {t.name} has shape {list(t.shape)}, expected {list(shape)}")

    def linear(t: Tensor, inn: int, out: int) -> np.ndarray:
        if t.dtype in _BLOCK:
            expect(t, (out, inn))
        elif t.dtype in (F32, F16):  # tensor_wmat: F16 -> WMat.h (load_weights.h:30-36)
            expect(t, (inn, out))
        else:
            raise BFileError(f"{path}: {t.name} is {DTYPE_NAMES.get(t.dtype, t.dtype)}; this device path runs "
                             "Q8_0, Q4_K, Q5_K, Q6_K, f16 and f32 weights")
        return t.array()

    def norm(key: str) -> np.ndarray:
        t = need(key)
        if t.dtype != F32:
            raise BFileError(f"{path}: {key} must be f32")
        expect(t, (D,))
        return t.array()

    dims = {"q": (D, qd), "k": (D, kvd), "v": (D, kvd), "o": (qd, D), "gate": (D, F), "up": (D, F), "down": (F, D)}
    wdt = need(layer_name(0, LAYER_SUFFIX["q"])).dtype
    ts: dict = {}
    qtypes: dict = {}  # K-quant tensors: their block type for the descriptor
    kinds = set()
    for l in range(L):
        ts[f"rms1.{l}"] = norm(layer_name(l, LAYER_SUFFIX["rms1"]))
        ts[f"rms2.{l}"] = norm(layer_name(l, LAYER_SUFFIX["rms2"]))
        for key, (inn, out) in dims.items():
            t = need(layer_name(l, LAYER_SUFFIX[key]))
            ts[f"{key}.{l}"] = linear(t, inn, out)
            kinds.add(t.dtype)
            if t.dtype in _KQ_CODE:
                qtypes[f"{key}.{l}"] = _KQ_CODE[t.dtype]
    # Q8_0 runs on its own kernels and cannot mix; f32 and the K-quants mix
    # freely (a mix is dequantised to f32 on the device)
    if Q8_0 in kinds and len(kinds) > 1:
        raise BFileError(f"{path}: Q8_0 linear weights mixed with {sorted(DTYPE_NAMES[k] for k in kinds - {Q8_0})}; "
                         "the device path runs Q8_0 models alone")
    if F16 in kinds and len(kinds) > 1:  # fp16 runs on its own GEMV variant
        raise BFileError(f"{path}: f16 linear weights mixed with {sorted(DTYPE_NAMES[k] for k in kinds - {F16})}; "
                         "the device path runs f16 models alone")
    # biases: bind_biases decides by layer 0's q bias (load_weights.h:128-136)
    qkv_bias = bf.get(layer_name(0, BIAS_SUFFIX["bq"])) is not None
    if qkv_bias:
        for l in range(L):
            for key, n in (("bq", qd), ("bk", kvd), ("bv", kvd)):
                t = need(layer_name(l, BIAS_SUFFIX[key]))
                if t.dtype != F32:
                    raise BFileError(f"{path}: {t.name} must be f32")
                expect(t, (n,))
                ts[f"{key}.{l}"] = t.array()
    emb = need("model.embed_tokens.weight")
    expect(emb, (V, D))
    if emb.dtype not in (F32, F16) + tuple(_BLOCK):
        raise BFileError(f"{path}: model.embed_tokens.weight is {DTYPE_NAMES.get(emb.dtype)}; the device path "
                         "reads f32, f16, Q8_0 or K-quant embeddings")
    head = bf.get("lm_head.weight")
    tied = head is None
    if tied:
        head = emb  # bind_lm_head's fallback (load_weights.h:142-144)
    if head.dtype in _BLOCK:
        if head.shape != (V, D):
            raise BFileError(f"{path}: {head.name} must be [vocab, hidden] = [{V}, {D}]")
    elif head.dtype in (F32, F16):  # bind_lm_head (load_weights.h:142-155)
        if head.shape != (D, V):
            raise BFileError(f"{path}: lm_head.weight missing or not [hidden, vocab] = [{D}, {V}]")
    else:
        raise BFileError(f"{path}: {head.name} is {DTYPE_NAMES.get(head.dtype)}; the device path runs Q8_0, "
                         "K-quant, f16 and f32")
    ts["head"] = head.array()
    if head.dtype in _KQ_CODE:
        qtypes["head"] = _KQ_CODE[head.dtype]
    if tied:
        embed = "tied"
    else:
        embed = {F32: "f32", F16: "f16"}.get(emb.dtype, "q8")  # "q8": a separate block-quantised embedding
        ts["embed"] = emb.array()
        if emb.dtype in _KQ_CODE:
            qtypes["embed"] = _KQ_CODE[emb.dtype]
    ts["final_norm"] = norm("model.norm.weight")
    if max_seq <= 0:
        max_seq = min(max(_info_int(info, "max_position_embeddings", 1024), 64), 4096)
    theta = float(_info_int(info, "rope_theta", 10000))
    wtype = "q8" if wdt == Q8_0 else "f16" if wdt == F16 else "kq" if kinds & set(_KQ_CODE) else "f32"
    cfg = Config(name or os.path.basename(os.path.normpath(path)), D, L, H, KV, hd, F, V, theta,
                 wtype, embed, qkv_bias, max_seq)
    cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
    hw = HostWeights(cfg, ts, cos, sin, qtypes=qtypes)
    hw.bfile = bf  # keeps the mapping alive with the views
    return hw


def model_dir_tensors(hw: HostWeights) -> tuple[dict, list]:
    """The header and tensor list (name, dtype, shape, bytes) of `hw` in the
    reference's names and layouts (Q8_0 [out, in], f32 / f16 [in, out]), in the
    order the reference's converter writes a model: embedding, final norm,
    per layer the nine weights (+ biases), lm_head unless tied."""
    cfg = hw.cfg
    D, F, V, qd, kvd = cfg.hidden, cfg.inter, cfg.vocab, cfg.q_dim, cfg.kv_dim
    header = dict(hidden=D, layers=cfg.layers, mode=1, num_heads=cfg.heads, num_kv_heads=cfg.kv_heads,
                  head_dim=cfg.head_dim, intermediate=F, vocab=V)

    def block_dtype(key: str) -> int:  # bfile dtype of a uint8 (block-quantised) tensor
        return _KQ_FILE.get(hw.qt.get(key, -1), Q8_0)

    def plain(a: np.ndarray) -> int:  # bfile dtype of an [in, out] tensor
        return F16 if a.dtype == np.uint16 else F32

    def lin(key: str, inn: int, out: int):
        a = hw.t[key]
        return (block_dtype(key), (out, inn), a) if a.dtype == np.uint8 else (plain(a), (inn, out), a)

    ts = []
    emb_key = "head" if cfg.embed == "tied" else "embed"
    emb = hw.t[emb_key]
    ts.append(("model.embed_tokens.weight", block_dtype(emb_key) if emb.dtype == np.uint8 else plain(emb), (V, D),
               emb))
    ts.append(("model.norm.weight", F32, (D,), hw.t["final_norm"]))
    dims = {"q": (D, qd), "k": (D, kvd), "v": (D, kvd), "o": (qd, D), "gate": (D, F), "down": (F, D), "up": (D, F)}
    for l in range(cfg.layers):
        for key in ("rms1", "q", "k", "v", "o", "rms2", "gate", "down", "up"):
            nm = layer_name(l, LAYER_SUFFIX[key])
            if key.startswith("rms"):
                ts.append((nm, F32, (D,), hw.t[f"{key}.{l}"]))
            else:
                dt, shape, a = lin(f"{key}.{l}", *dims[key])
                ts.append((nm, dt, shape, a))
        if cfg.qkv_bias:
            for key, n in (("bq", qd), ("bk", kvd), ("bv", kvd)):
                ts.append((layer_name(l, BIAS_SUFFIX[key]), F32, (n,), hw.t[f"{key}.{l}"]))
    if cfg.embed != "tied":
        h = hw.t["head"]
        ts.append(("lm_head.weight",) + ((block_dtype("head"), (V, D), h) if h.dtype == np.uint8
                                         else (plain(h), (D, V), h)))
    return header, ts


def save_model_dir(hw: HostWeights, path: str) -> None:
    """Writes `hw` as a reference model directory (model.bf +
    model_info.json with the keys the reference's own writer emits,
    libs/text/text.h:653-662)."""
    os.makedirs(path, exist_ok=True)
    header, ts = model_dir_tensors(hw)
    write_bfile(os.path.join(path, "model.bf"), header, ts)
    cfg = hw.cfg
    info = {"hidden_size": str(cfg.hidden), "layer_count": str(cfg.layers), "num_heads": str(cfg.heads),
            "num_kv_heads": str(cfg.kv_heads), "head_dim": str(cfg.head_dim),
            "intermediate_size": str(cfg.inter), "vocab_size": str(cfg.vocab),
            "rope_theta": str(int(cfg.theta)), "max_position_embeddings": str(cfg.max_seq)}
    with open(os.path.join(path, "model_info.json"), "w", encoding="utf-8") as f:
        json.dump(info, f, indent=1)


__all__ = ["BFile", "BFileError", "Tensor", "write_bfile", "load_model_dir", "save_model_dir",
           "model_dir_tensors", "tensor_bytes"]
