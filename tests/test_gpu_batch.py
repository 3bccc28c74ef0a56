"""Batched decode (jyc_batch_*): B sequences with ragged prompts decoded
together must each follow the reference's greedy sequence for its own prompt.

Every token a sequence appends is replayed through the oracle (bit-identical
to the reference's forward, tests/test_oracle_golden.py) on that sequence's
own history: it must be the oracle's argmax, or the oracle's top-2 logit gap
at that step must be a near tie (below twice LOGIT_TOL of max|logit|, the
bar of the model tests). B <= 8 runs the few-row matmul (RMSNorm fused),
B >= 9 the tcgen05 token tiles (B = 12 pads one 16-row tile, B = 20 pads the
last of two).
"""
import ctypes as C

import numpy as np
import pytest

from _util import LOGIT_TOL, ptr
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, BatchDecoder, DeviceModel, HostWeights, synth_ids

pytestmark = pytest.mark.gpu

STEPS = 10


@pytest.fixture(scope="module")
def c0(cuda):
    hw = HostWeights.synthetic(CONFIGS["c0"])
    m = DeviceModel(hw)
    yield hw, m
    m.close()


def _prompts(cfg, n):
    lens = [17 + (7 * b) % 32 for b in range(n)]
    return [synth_ids(91, 1000 + b, cfg.vocab, ln) for b, ln in enumerate(lens)]


def _replay(oracle, hw, seq, prompt_len):
    """(mismatches, near_ties) of the device's generated tokens against the
    oracle's argmax on the same history."""
    cfg = hw.cfg
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    want = np.empty(cfg.vocab, np.float32)
    bad, ties = [], 0
    try:
        tok = np.ascontiguousarray(seq[:prompt_len], np.int32)
        pos = 0
        for i in range(prompt_len, len(seq)):
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(tok), len(tok), pos, ptr(want), None) == 0
            pos += len(tok)
            best = int(np.argmax(want))
            if seq[i] != best:
                top2 = np.sort(want)[-2:]
                if top2[1] - top2[0] < 2 * LOGIT_TOL * np.abs(want).max():
                    ties += 1
                else:
                    bad.append((i, int(seq[i]), best))
            tok = np.array([seq[i]], np.int32)
    finally:
        oracle.cache_free(cache)
    return bad, ties


@pytest.mark.parametrize("nseq,path", [(2, 1), (4, 1), (7, 1), (8, 1), (12, 2), (16, 2), (20, 2)])
def test_batch_follows_reference_per_sequence(c0, oracle, nseq, path):
    hw, m = c0
    prompts = _prompts(hw.cfg, nseq)
    bt = BatchDecoder(m, nseq)
    try:
        assert bt.path() == path
        for b, p in enumerate(prompts):
            bt.prefill(b, p)
        launches = _capi.load().jyc_kernel_launches()
        bt.decode(STEPS)
        assert _capi.load().jyc_kernel_launches() - launches == STEPS * bt.kernels_per_step()
        assert _capi.load().jyc_device_error(1) == 0
        total_ties = 0
        for b, p in enumerate(prompts):
            seq = bt.tokens(b)
            assert len(seq) == len(p) + 1 + STEPS
            assert np.array_equal(seq[:len(p)], p)
            bad, ties = _replay(oracle, hw, seq, len(p))
            assert not bad, f"sequence {b}: (position, device, oracle) {bad}"
            total_ties += ties
        assert total_ties <= max(1, nseq * STEPS // 20)
    finally:
        bt.close()


@pytest.mark.parametrize("nseq", [6, 16])
def test_batch_rewind_replays_identically(c0, nseq):
    hw, m = c0
    prompts = [synth_ids(92, 7 + b, hw.cfg.vocab, 24) for b in range(nseq)]
    bt = BatchDecoder(m, nseq)
    try:
        for b, p in enumerate(prompts):
            bt.prefill(b, p)
        bt.decode(6)
        first = [bt.tokens(b) for b in range(nseq)]
        bt.rewind(25)
        bt.decode(6)
        again = [bt.tokens(b) for b in range(nseq)]
        for a, g in zip(first, again):
            assert np.array_equal(a, g)
    finally:
        bt.close()


def test_batch_rejects_bad_arguments(c0):
    hw, m = c0
    lib = _capi.load()
    assert not lib.jyc_batch_create(m.h, 0)
    assert not lib.jyc_batch_create(m.h, 100000)
    bt = BatchDecoder(m, 2)
    try:
        p = np.arange(5, dtype=np.int32)
        assert lib.jyc_batch_prefill(bt.h, 2, p.ctypes.data, 5) == _capi.JYC_ERR_ARG
        assert lib.jyc_batch_prefill(bt.h, 0, p.ctypes.data, hw.cfg.max_seq) == _capi.JYC_ERR_ARG
        assert lib.jyc_batch_rewind(bt.h, 0, None) == _capi.JYC_ERR_ARG
    finally:
        bt.close()
