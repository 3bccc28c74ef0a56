"""The reference arm of bench.py builds its seeded model with liboracle.so
(oracle.synth), without the product library: its bytes, descriptor layout,
RoPE tables and prompt ids must equal the library's (jyc_synth_*,
HostWeights.synthetic, prompt_ids), so both arms time the same model."""
import ctypes as C

import numpy as np

from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, HostWeights, prompt_ids
from oracle import synth


def test_generators_byte_identical(oracle):
    lib = _capi.load()
    o = oracle.lib
    o.jyo_synth_f32.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_size_t]
    o.jyo_synth_q8_0.argtypes = [C.c_uint64, C.c_uint64, C.c_float, C.c_void_p, C.c_size_t, C.c_size_t]
    o.jyo_synth_ids.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_void_p, C.c_size_t]
    for seed, stream, std in ((1234, 7, 0.02), (5, 1 << 20, 1.5), (2 ** 40 + 3, 99, 1e-6)):
        a = np.empty(4099, np.float32)
        b = np.empty_like(a)
        lib.jyc_synth_f32(seed, stream, std, a.ctypes.data, a.size)
        o.jyo_synth_f32(seed, stream, std, b.ctypes.data, b.size)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        rows, k = 37, 320
        qa = np.empty(rows * (k // 32) * 34, np.uint8)
        qb = np.empty_like(qa)
        lib.jyc_synth_q8_0(seed, stream, std, qa.ctypes.data, rows, k)
        o.jyo_synth_q8_0(seed, stream, std, qb.ctypes.data, rows, k)
        assert np.array_equal(qa, qb)
        ia = np.empty(1000, np.int32)
        ib = np.empty_like(ia)
        lib.jyc_synth_ids(seed, stream, 151936, ia.ctypes.data, ia.size)
        o.jyo_synth_ids(seed, stream, 151936, ib.ctypes.data, ib.size)
        assert np.array_equal(ia, ib)


def test_structures_match_the_header_layout():
    for mine, lib in ((synth.WMat, _capi.WMat), (synth.LayerWeights, _capi.LayerWeights),
                      (synth.ModelDesc, _capi.ModelDesc)):
        assert C.sizeof(mine) == C.sizeof(lib)
        assert [(f, getattr(mine, f).offset) for f, _ in mine._fields_] == \
               [(f, getattr(lib, f).offset) for f, _ in lib._fields_]


def test_synth_model_equals_host_weights(oracle):
    """configs[1] (tied embedding, QKV bias): every tensor, the RoPE tables
    and the prompt ids equal the library's."""
    cfg = CONFIGS["c1"]
    hw = HostWeights.synthetic(cfg)
    sm = synth.SynthModel(synth.SHAPES["c1"], cfg.max_seq, oracle=oracle)
    for l in (0, cfg.layers - 1):
        for n in ("q", "k", "v", "o", "gate", "up", "down", "bq", "bk", "bv"):
            assert np.array_equal(hw.t[f"{n}.{l}"], sm.t[f"{n}.{l}"]), (n, l)
    assert np.array_equal(hw.t["head"], sm.t["head"])
    assert np.array_equal(hw.cos, sm.cos) and np.array_equal(hw.sin, sm.sin)
    assert np.array_equal(prompt_ids(cfg, n=512), synth.prompt(oracle, cfg.vocab, 512))
    assert sm.weight_bytes_per_token() == hw.weight_bytes_per_token()
    d, e = sm.desc, hw.desc
    for f in ("num_layers", "max_seq", "vocab_size", "hidden", "num_heads", "num_kv_heads", "head_dim",
              "intermediate"):
        assert getattr(d, f) == getattr(e, f), f


def test_f16_weights_are_the_fp32_ones_rounded():
    """synthetic_f16: every linear matrix, the LM head and the embedding are the
    seeded fp32 weights rounded to IEEE halves ([in][out] layout kept), bound
    through WMat.h; norms stay fp32."""
    from dataclasses import replace
    cfg = replace(CONFIGS["c0"], layers=2)
    f32 = HostWeights.synthetic(replace(cfg, wtype="f32", embed="f32"))
    f16 = HostWeights.synthetic_f16(cfg)
    assert f16.cfg.wtype == "f16" and f16.cfg.embed == "f16"
    for key, a in f16.t.items():
        if key.split(".")[0] in ("q", "k", "v", "o", "gate", "up", "down", "head", "embed"):
            assert a.dtype == np.uint16
            assert np.array_equal(a, f32.t[key].astype(np.float16).view(np.uint16)), key
        else:
            assert np.array_equal(a, f32.t[key]), key
    lw = f16.desc.layers[0]
    assert lw.Wq.h and not lw.Wq.f and not lw.Wq.q
    assert f16.desc.lm_head.h and f16.desc.embed.h
    lin = (cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim + 3 * cfg.inter * cfg.hidden
    want = cfg.layers * (2.0 * lin + 2 * cfg.hidden * 4) + cfg.vocab * cfg.hidden * 2.0 + 4 * cfg.hidden + cfg.hidden * 4
    assert f16.weight_bytes_per_token() == want
