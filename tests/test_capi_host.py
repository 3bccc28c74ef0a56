"""CPU: the C-ABI library loads, exports every entry point include/jieyu_b200.h
declares, and its host-side helpers (RoPE tables, seeded synthetic data,
Q8_0 quantiser) behave. No kernel is launched here."""
import os
import re

import numpy as np

from _util import golden, ptr, sha
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, quantize_q8, rope_table, synth_f32, synth_ids, synth_q8

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"JYC_API\s+[^;(]*?\b(jyc_\w+)\s*\(", src)
            names += re.findall(r"JIEYU_API\s+[^;(]*?\b((?:jieyu|jyt)_\w+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    names = declared_symbols()
    assert len(names) >= 30 and "jieyu_generate" in names and "jyt_tok_encode" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    bound = {n for n, _, _ in _capi.SIGNATURES}
    assert set(names) <= bound, sorted(set(names) - bound)


def test_version_and_errors():
    lib = _capi.load()
    assert b"sm_100a" in lib.jyc_version()
    assert lib.jyc_synth_q8_0(1, 2, 0.02, None, 4, 33) == _capi.JYC_ERR_ARG
    assert "multiple of 32" in _capi.last_error()


def test_rope_tables_equal_reference():
    g = golden("host.json")
    for key in ("c0", "c1", "c2", "c3"):
        c = CONFIGS[key]
        cs, sn = rope_table(c.max_seq, c.head_dim, c.theta)
        assert sha(np.concatenate([cs, sn])) == g[f"rope_{key}"], key


def test_synthetic_generator_is_pinned():
    g = golden("host.json")
    assert sha(synth_q8(1234, 5, 64, 512)) == g["synth_q8"]
    assert sha(synth_f32(1234, 6, 4096)) == g["synth_f32"]
    ids = synth_ids(1234, 7, 151936, 1000)
    assert sha(ids) == g["synth_ids"]
    assert ids.min() >= 0 and ids.max() < 151936


def test_synthetic_statistics():
    x = synth_f32(5, 9, 200_000, 0.02)
    assert abs(x.mean()) < 2e-4 and abs(x.std() - 0.02) < 4e-4


def _dequant(blocks, rows, k):
    b = blocks.reshape(rows, k // 32, 34)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, :, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(rows, k)


def test_quantizer_round_trip_and_edges():
    rows, k = 16, 256
    x = synth_f32(3, 4, rows * k, 1.0).reshape(rows, k)
    x[0, :32] = 0.0                 # all-zero block -> d = 0, q = 0
    x[1, :32] = 1e-30               # far below fp16 range -> d = 0
    x[2, 5] = 65504.0 * 127         # overflow to d = inf is avoided: d = fp16(amax/127)
    blocks = quantize_q8(x, rows, k)
    y = _dequant(blocks, rows, k)
    assert np.all(y[0, :32] == 0)
    d = blocks.reshape(rows, k // 32, 34)[:, :, :2].copy().view(np.float16).astype(np.float32)[..., 0]
    err = np.abs(y - x).reshape(rows, k // 32, 32).max(axis=2)
    # half a quantisation step (plus the clamp at 127 after fp16 rounding of d)
    assert np.all(err[2:] <= d[2:] * 0.51)
    q = blocks.reshape(rows, k // 32, 34)[:, :, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
