"""Model directories (jieyu_b200.bfile) against the reference's own code, on
the CPU.

* `write_bfile` writes the same bytes as the reference's bfile::write_bfile
  (libs/model_libs/bfile.h:275-343, compiled from its sources into
  oracle/_ref) for the same header and tensors;
* the reference's reader and binder (View::open, bfile.h:141-176; bind_layers /
  bind_biases / bind_embed / bind_lm_head / bind_final_norm,
  load_weights.h:97-155) take every weight from the same bytes of the file
  as `load_model_dir`, including the tied-head fallback;
* files the reference's reader rejects (magic, version, entry size, data
  offset, misaligned or overlong tensors, dimension count, dtype, size
  mismatch) are rejected here too, and the binding errors of bind_model
  (pipeline.h:63-153: missing tensors, transposed shapes) are raised;
* a written directory loads back to the same host tensors and config,
  including a model in the K-quant formats (Q4_K / Q5_K / Q6_K mixed per
  matrix) that the reference's downloads use.
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

from jieyu_b200 import bfile
from jieyu_b200.model import Config, HostWeights
from oracle.bind import REF_SO

TINY_Q8_TIED = Config("tiny_q8_tied", 64, 2, 4, 2, 16, 96, 100, 1e6, "q8", "tied", True, 128)
TINY_Q8 = Config("tiny_q8", 64, 2, 4, 1, 16, 96, 100, 5e5, "q8", "q8", False, 128)
TINY_F32 = Config("tiny_f32", 32, 1, 2, 1, 8, 64, 50, 1e4, "f32", "f32", False, 64)


def _models():
    from _kquant import kquant_model
    return {
        "bind_kat": HostWeights.bind_test_kat(),
        "q8_tied_bias": HostWeights.synthetic(TINY_Q8_TIED, seed=5),
        "q8_separate": HostWeights.synthetic(TINY_Q8, seed=6),
        "f32_rect": HostWeights.synthetic(TINY_F32, seed=7),
        "f16_rect": HostWeights.synthetic_f16(TINY_F32, seed=8),
        "kquant_mixed": kquant_model(),
    }


MODELS = list(_models())


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_SO):
        pytest.skip("reference harness not built (reference tree absent)")
    lib = C.CDLL(REF_SO)
    P = C.c_void_p
    lib.jyref_bfile_write.restype = C.c_int
    lib.jyref_bfile_write.argtypes = [C.c_char_p, P, C.c_int, P, P, P, P, P, P]
    lib.jyref_bfile_bind.restype = C.c_int
    lib.jyref_bfile_bind.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, P, P]
    lib.jyref_last_error.restype = C.c_char_p
    return lib


def _ref_write(lib, path, header, tensors):
    n = len(tensors)
    hdr = np.array([header["hidden"], header["layers"], header.get("mode", 1), header["num_heads"],
                    header["num_kv_heads"], header["head_dim"], header["intermediate"], header["vocab"]],
                   dtype=np.uint64)
    names = (C.c_char_p * n)(*[t[0].encode() for t in tensors])
    dtypes = np.array([t[1] for t in tensors], dtype=np.uint8)
    ndims = np.array([len(t[2]) for t in tensors], dtype=np.uint8)
    shapes = np.zeros((n, 4), dtype=np.uint32)
    for i, t in enumerate(tensors):
        shapes[i, :len(t[2])] = t[2]
    arrs = [np.ascontiguousarray(t[3]) for t in tensors]
    data = (C.c_void_p * n)(*[a.ctypes.data for a in arrs])
    nbytes = np.array([a.nbytes for a in arrs], dtype=np.uint64)
    r = lib.jyref_bfile_write(path.encode(), hdr.ctypes.data, n, C.cast(names, C.c_void_p), dtypes.ctypes.data,
                              ndims.ctypes.data, shapes.ctypes.data, C.cast(data, C.c_void_p), nbytes.ctypes.data)
    assert r == 0, lib.jyref_last_error()


def _ref_bind(lib, path, cfg):
    L = cfg.layers
    out = np.zeros(12 * L + 3, dtype=np.int64)
    dt = np.zeros(12 * L + 3, dtype=np.uint8)
    r = lib.jyref_bfile_bind(path.encode(), L, cfg.hidden, cfg.vocab, out.ctypes.data, dt.ctypes.data)
    return r, out, dt


def _save(hw, d):
    bfile.save_model_dir(hw, str(d))
    return os.path.join(str(d), "model.bf")


@pytest.mark.parametrize("model", MODELS)
def test_writer_matches_reference_bytes(ref, tmp_path, model):
    hw = _models()[model]
    header, ts = bfile.model_dir_tensors(hw)
    ours, theirs = str(tmp_path / "ours.bf"), str(tmp_path / "ref.bf")
    bfile.write_bfile(ours, header, ts)
    _ref_write(ref, theirs, header, ts)
    a, b = open(ours, "rb").read(), open(theirs, "rb").read()
    assert len(a) == len(b) and a == b


@pytest.mark.parametrize("model", MODELS)
def test_reference_binds_the_same_bytes(ref, tmp_path, model):
    hw = _models()[model]
    path = _save(hw, tmp_path)
    got = bfile.load_model_dir(str(tmp_path), max_seq=hw.cfg.max_seq)
    r, out, dt = _ref_bind(ref, path, hw.cfg)
    assert r == 0, ref.jyref_last_error()
    base = got.bfile.map.ctypes.data

    def off(key):
        return got.t[key].ctypes.data - base if key in got.t else -1

    L = hw.cfg.layers
    order = ["rms1", "q", "k", "v", "o", "rms2", "gate", "down", "up", "bq", "bk", "bv"]
    for l in range(L):
        for k, key in enumerate(order):
            assert out[12 * l + k] == off(f"{key}.{l}"), (l, key)
            if out[12 * l + k] >= 0 and key in ("q", "k", "v", "o", "gate", "down", "up"):
                name = f"{key}.{l}"
                if name in hw.qt:
                    want = {0: bfile.Q4K, 1: bfile.Q5K, 2: bfile.Q6K}[hw.qt[name]]
                else:
                    want = {"q8": bfile.Q8_0, "f16": bfile.F16}.get(hw.cfg.wtype, bfile.F32)
                assert dt[12 * l + k] == want
    emb_key = "head" if hw.cfg.embed == "tied" else "embed"
    assert out[12 * L] == off(emb_key)
    assert out[12 * L + 1] == off("head")  # lm_head.weight, or the tied embedding
    assert out[12 * L + 2] == off("final_norm")


@pytest.mark.parametrize("model", MODELS)
def test_directory_round_trip(tmp_path, model):
    hw = _models()[model]
    _save(hw, tmp_path)
    got = bfile.load_model_dir(str(tmp_path), max_seq=hw.cfg.max_seq)
    for f in ("hidden", "layers", "heads", "kv_heads", "head_dim", "inter", "vocab", "wtype", "embed",
              "qkv_bias", "max_seq"):
        assert getattr(got.cfg, f) == getattr(hw.cfg, f), f
    assert got.cfg.theta == float(int(hw.cfg.theta))
    assert set(got.t) == set(hw.t)
    assert got.qt == hw.qt
    for k in hw.t:
        a, b = np.asarray(hw.t[k]), np.asarray(got.t[k])
        assert a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8)), k
    assert np.array_equal(got.cos, hw.cos) and np.array_equal(got.sin, hw.sin)


def _patch(path, offset, data):
    with open(path, "r+b") as f:
        f.seek(offset)
        f.write(data)


def _entry_field(i, field):
    base = bfile.HEADER + i * bfile.ENTRY
    return base + {"dtype": 64, "ndim": 65, "shape0": 68, "offset": 88, "nbytes": 96}[field]


CORRUPT = {
    "magic": lambda p, n: _patch(p, 0, b"JYAIBX"),
    "version1": lambda p, n: _patch(p, 38, (1).to_bytes(4, "little")),
    "entry_size": lambda p, n: _patch(p, 50, (100).to_bytes(4, "little")),
    "data_off_past_end": lambda p, n: _patch(p, 46, (n + 64).to_bytes(4, "little")),
    "directory_too_long": lambda p, n: _patch(p, 42, (10_000).to_bytes(4, "little")),
    "misaligned_tensor": lambda p, n: _patch(p, _entry_field(1, "offset"), (32).to_bytes(8, "little")),
    "nbytes_mismatch": lambda p, n: _patch(p, _entry_field(0, "nbytes"), (12).to_bytes(8, "little")),
    "five_dims": lambda p, n: _patch(p, _entry_field(0, "ndim"), bytes([5])),
    "unknown_dtype": lambda p, n: _patch(p, _entry_field(0, "dtype"), bytes([42])),
    "truncated": lambda p, n: os.truncate(p, n - 8),
}


@pytest.mark.parametrize("how", list(CORRUPT))
def test_rejects_what_the_reference_rejects(ref, tmp_path, how):
    hw = _models()["q8_tied_bias"]
    path = _save(hw, tmp_path)
    CORRUPT[how](path, os.path.getsize(path))
    r, _, _ = _ref_bind(ref, path, hw.cfg)
    assert r == 1, f"the reference's reader accepted {how}"
    with pytest.raises(bfile.BFileError):
        bfile.BFile(path)


def _write_dir(d, hw, edit):
    header, ts = bfile.model_dir_tensors(hw)
    ts = edit(ts)
    os.makedirs(d, exist_ok=True)
    bfile.write_bfile(os.path.join(d, "model.bf"), header, ts)
    with open(os.path.join(d, "model_info.json"), "w") as f:
        json.dump({"rope_theta": "10000", "max_position_embeddings": "64"}, f)


def test_binding_errors(ref, tmp_path):
    hw = _models()["f32_rect"]
    cfg = hw.cfg
    # a missing weight: the reference's bind_layers fails too
    d = str(tmp_path / "missing")
    _write_dir(d, hw, lambda ts: [t for t in ts if t[0] != "model.layers.0.mlp.up_proj.weight"])
    assert _ref_bind(ref, os.path.join(d, "model.bf"), cfg)[0] == 2
    with pytest.raises(bfile.BFileError, match="mlp.up_proj"):
        bfile.load_model_dir(d)
    # q_proj stored [out, in] in f32 (bind_model's "2D weights need transposing")
    d = str(tmp_path / "transposed")
    q = "model.layers.0.self_attn.q_proj.weight"
    _write_dir(d, hw, lambda ts: [(n, dt, tuple(reversed(s)) if n == q else s, a) for n, dt, s, a in ts])
    with pytest.raises(bfile.BFileError, match="q_proj"):
        bfile.load_model_dir(d)
    # no final norm
    d = str(tmp_path / "nonorm")
    _write_dir(d, hw, lambda ts: [t for t in ts if t[0] != "model.norm.weight"])
    with pytest.raises(bfile.BFileError, match="model.norm.weight"):
        bfile.load_model_dir(d)
    # one f16 weight among f32 ones: valid for the reference, a mix this device
    # path does not run (fp16 models decode with all linear weights in fp16)
    d = str(tmp_path / "f16")
    o = "model.layers.0.self_attn.o_proj.weight"
    _write_dir(d, hw, lambda ts: [(n, bfile.F16, s, np.zeros(int(np.prod(s)), np.uint16)) if n == o
                                  else (n, dt, s, a) for n, dt, s, a in ts])
    assert _ref_bind(ref, os.path.join(d, "model.bf"), cfg)[0] == 0
    with pytest.raises(bfile.BFileError, match="f16"):
        bfile.load_model_dir(d)
    # no model_info.json
    os.remove(os.path.join(d, "model_info.json"))
    with pytest.raises(bfile.BFileError, match="model_info.json"):
        bfile.load_model_dir(d)


@pytest.mark.parametrize("info,want", [({"max_position_embeddings": "100000"}, 4096),
                                       ({"max_position_embeddings": 10}, 64),
                                       ({"max_position_embeddings": "2048"}, 2048), ({}, 1024)])
def test_max_seq_from_model_info(tmp_path, info, want):
    hw = _models()["f32_rect"]
    _save(hw, tmp_path)
    with open(tmp_path / "model_info.json", "w") as f:
        json.dump(info, f)
    got = bfile.load_model_dir(str(tmp_path))
    assert got.cfg.max_seq == want and got.cfg.theta == 10000.0
