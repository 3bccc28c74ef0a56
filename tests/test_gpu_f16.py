"""fp16 weights on the device (matmul_f16.h, WMat.h): the operator entry
points (jyc_matmul_f16 over device buffers, jyc_host_matmul_f16 and the
matmul_w dispatch over host buffers) against the oracle, which is pinned to
the reference's own matmul_f16 (tests/golden/f16.json); and a configs[0]-shaped
model with every linear matrix, the LM head and the embedding in fp16 decoding
on the generic kernels (2 bytes per weight streamed) against the oracle.

Bars: matmuls within 2e-5 of max|y| (fp32 sums in another order; the fp16 ->
fp32 conversion is exact on both sides); model logits within 1e-3 of
max|logit| per teacher-forced step; the greedy sequence equal to the
reference's (golden) wherever the reference's top-2 gap is not a near tie.
"""
import ctypes as C
import os
import sys

import numpy as np
import pytest

from _util import LOGIT_TOL, dev, golden, ptr, stream
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden_f16 as mgf  # noqa: E402

pytestmark = pytest.mark.gpu

SHAPES = mgf.F16_CASES + [(8, 896, 4864), (12, 257, 64), (16, 512, 1376), (1, 32000, 512)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matmul_f16_device(cuda, oracle, m, n, k):
    torch = cuda
    lib = _capi.load()
    a, b = mgf.f16_inputs(m, n, k)
    want = np.empty(m * n, np.float32)
    oracle.matmul_f16(ptr(a), ptr(b), ptr(want), m, n, k)
    da, db = dev(torch, a), dev(torch, b.view(np.int16))
    dbt = torch.empty(k * n, dtype=torch.int16, device="cuda")
    dc = torch.empty(m * n, dtype=torch.float32, device="cuda")
    s = stream(torch)
    _capi.check(lib.jyc_f16_transpose(db.data_ptr(), dbt.data_ptr(), k, n, s))
    _capi.check(lib.jyc_matmul_f16(da.data_ptr(), dbt.data_ptr(), dc.data_ptr(), m, n, k, s))
    got = dc.cpu().numpy()
    amax = max(np.abs(want).max(), 1e-30)
    assert np.abs(got - want).max() <= 2e-5 * amax
    # deterministic: a second call gives the same bits
    _capi.check(lib.jyc_matmul_f16(da.data_ptr(), dbt.data_ptr(), dc.data_ptr(), m, n, k, s))
    assert np.array_equal(dc.cpu().numpy().view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(1, 64, 512), (2, 13, 5), (9, 100, 72)])
def test_matmul_f16_host_and_matmul_w(cuda, oracle, m, n, k):
    lib = _capi.load()
    a, b = mgf.f16_inputs(m, n, k)
    want = np.empty(m * n, np.float32)
    oracle.matmul_f16(ptr(a), ptr(b), ptr(want), m, n, k)
    amax = max(np.abs(want).max(), 1e-30)
    got = np.empty(m * n, np.float32)
    _capi.check(lib.jyc_host_matmul_f16(ptr(a), ptr(b), ptr(got), m, n, k))
    assert np.abs(got - want).max() <= 2e-5 * amax
    w = _capi.WMat(None, ptr(b), None, 0)
    got2 = np.empty(m * n, np.float32)
    _capi.check(lib.jyc_host_matmul_w(C.byref(w), m, n, k, ptr(a), ptr(got2)))
    assert np.array_equal(got2.view(np.uint32), got.view(np.uint32))


@pytest.fixture(scope="module")
def c0_f16(cuda):
    hw = HostWeights.synthetic_f16(CONFIGS["c0"])
    m = DeviceModel(hw)
    yield hw, m
    m.close()


def test_f16_model_uses_the_generic_path_at_2_bytes_per_weight(c0_f16):
    hw, m = c0_f16
    lib = _capi.load()
    assert lib.jyc_model_decode_path(m.h) == 0
    assert abs(lib.jyc_model_weight_bytes_per_token(m.h) - hw.weight_bytes_per_token()) < 1e-6 * hw.weight_bytes_per_token()


def test_f16_model_teacher_forced_logits(c0_f16, oracle):
    """16 decode steps fed the oracle's greedy tokens: device logits within
    1e-3 of max|logit| of the oracle's at every step."""
    hw, m = c0_f16
    cfg = hw.cfg
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    want = np.empty(cfg.vocab, np.float32)
    tok = np.ascontiguousarray(prompt_ids(cfg), np.int32)
    pos = 0
    try:
        for s in range(17):
            got = m.forward_logits(tok, pos)
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(tok), len(tok), pos, ptr(want), None) == 0
            amax = np.abs(want).max()
            err = np.abs(got - want).max()
            print(f"  f16 step {s}: max|dlogit|/max|logit| = {err / amax:.2e}")
            assert err <= LOGIT_TOL * amax
            pos += len(tok)
            tok = np.array([int(np.argmax(want))], np.int32)
    finally:
        oracle.cache_free(cache)


def test_f16_model_greedy_sequence(c0_f16):
    """The 64-token greedy sequence equals the reference's (golden)."""
    hw, m = c0_f16
    g = golden("f16.json")["c0_f16"]
    out = m.generate(np.array(g["prompt"], np.int32), 64)
    assert list(out) == g["greedy"]


def test_f16_model_directory_decodes_like_memory(cuda, tmp_path, c0_f16):
    """An fp16 model directory (model.bf with F16 tensors, bound by the
    reference's rules; tests/test_bfile_host.py pins the bytes and the
    binding) decodes the same greedy tokens as the same weights from memory."""
    from jieyu_b200 import bfile
    hw, m = c0_f16
    bfile.save_model_dir(hw, str(tmp_path))
    loaded = bfile.load_model_dir(str(tmp_path), max_seq=hw.cfg.max_seq)
    assert loaded.cfg.wtype == "f16" and loaded.cfg.embed == "f16"
    prompt = prompt_ids(hw.cfg, n=16)
    want = m.generate(prompt, 24)
    m2 = DeviceModel(loaded)
    try:
        got = m2.generate(prompt, 24)
    finally:
        m2.close()
    assert np.array_equal(got, want)
