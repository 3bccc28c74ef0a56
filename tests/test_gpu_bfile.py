"""Model directories on the device path: a reference model directory
(model.bf + model_info.json, the format of libs/model_libs/bfile.h; written
here by jieyu_b200.bfile, whose bytes tests/test_bfile_host.py pins to the
reference's own writer) loaded with load_model_dir and uploaded decodes the
same greedy tokens as the same weights bound from memory, and the
reference's check_bind_weights model (libs/text/text.h:817-843, the
directory its KAT writes) reproduces the KAT's golden ids from disk.
"""
import numpy as np
import pytest

from _util import golden
from jieyu_b200 import bfile
from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids

pytestmark = pytest.mark.gpu


def _generate(hw, prompt, n):
    m = DeviceModel(hw)
    try:
        return m.generate(prompt, n)
    finally:
        m.close()


@pytest.mark.parametrize("key", ["c0", "c1"])
def test_loaded_directory_decodes_like_memory(cuda, tmp_path, key):
    cfg = CONFIGS[key]
    if key == "c1":  # Qwen2.5-0.5B shape (tied Q8_0 head, QKV bias), 2 layers
        from dataclasses import replace
        cfg = replace(cfg, layers=2, max_seq=256, name="c1_2layer")
    hw = HostWeights.synthetic(cfg)
    bfile.save_model_dir(hw, str(tmp_path))
    loaded = bfile.load_model_dir(str(tmp_path), max_seq=cfg.max_seq)
    assert loaded.cfg.embed == cfg.embed and loaded.cfg.qkv_bias == cfg.qkv_bias
    prompt = prompt_ids(cfg, n=16)
    want = _generate(hw, prompt, 24)
    got = _generate(loaded, prompt, 24)
    assert np.array_equal(got, want)


def test_bind_kat_from_disk(cuda, tmp_path):
    g = golden("kat.json")
    bfile.save_model_dir(HostWeights.bind_test_kat(), str(tmp_path))
    hw = bfile.load_model_dir(str(tmp_path), max_seq=8)
    assert list(_generate(hw, np.array([1, 2, 3]), 3)) == g["bind_123"]
