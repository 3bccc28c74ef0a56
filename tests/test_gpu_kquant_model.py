"""A model in the reference's K-quant formats on the device path: Q4_K /
Q5_K / Q6_K weights (mixed per matrix, Q6_K head and embedding). The layer
matrices stay K-quant blocks on the device and the K-quant matmul reads them
in place (the head and embedding are dequantised once to fp32); the
comparison path (JYC_KQ_FP32=1) dequantises every matrix at upload and runs
the fp32 matmuls. Fed the same tokens, the device's logits must match the
oracle's (whose K-quant generate is bit-identical to the reference's,
tests/test_kquant_model_host.py) within the model tests' LOGIT_TOL, with the
same argmax wherever the oracle's top-2 gap is not a near tie; the same model
written as a reference model directory and loaded back decodes identically.
"""
import numpy as np
import pytest

from _kquant import kquant_model
from jieyu_b200 import _capi, bfile
from jieyu_b200.model import DeviceModel
from test_gpu_model import _check_logits, _teacher_forced

pytestmark = pytest.mark.gpu

PROMPT = np.array([3, 17, 255, 42, 7, 99, 150, 8], np.int32)


@pytest.mark.parametrize("path", ["in_place", "fp32"])
def test_kquant_model_logits_follow_the_oracle(cuda, oracle, monkeypatch, path):
    hw = kquant_model()
    if path == "fp32":
        monkeypatch.setenv("JYC_KQ_FP32", "1")
    m = DeviceModel(hw)
    monkeypatch.delenv("JYC_KQ_FP32", raising=False)
    try:
        lib = _capi.load()
        dev_bytes = lib.jyc_model_weight_bytes_per_token(m.h)
        if path == "in_place":  # the blocks' own bytes, not 4 B per weight
            assert abs(dev_bytes - hw.weight_bytes_per_token()) <= 1e-9 * dev_bytes
        rels = [_check_logits(got, want) for s, got, want, cache, n in _teacher_forced(m, hw, oracle, PROMPT, 8)]
    finally:
        m.close()
    assert max(rels) < 1e-3


def test_kquant_model_directory_decodes_like_memory(cuda, tmp_path):
    hw = kquant_model()
    bfile.save_model_dir(hw, str(tmp_path))
    loaded = bfile.load_model_dir(str(tmp_path), max_seq=hw.cfg.max_seq)
    assert loaded.cfg.wtype == "kq" and loaded.qt == hw.qt
    outs = []
    for w in (hw, loaded):
        m = DeviceModel(w)
        try:
            outs.append(m.generate(PROMPT, 12))
        finally:
            m.close()
    assert len(outs[0]) == len(PROMPT) + 12
    assert np.array_equal(outs[0], outs[1])
