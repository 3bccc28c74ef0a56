"""CPU: the oracle (plain-C restatement) reproduces the reference's own outputs
recorded in tests/golden (produced by tests/golden/make_golden.py running the
reference). These pin the checker the GPU tests trust."""
import ctypes as C
import os
import sys

import numpy as np
import pytest

from _util import golden, ptr, sha

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden  # noqa: E402

from jieyu_b200.model import CONFIGS, HostWeights, prompt_ids  # noqa: E402


def test_oracle_ops_match_reference_digests(oracle):
    want = golden("ops.json")["ops"]
    got = make_golden.run_ops(oracle)
    assert set(got) == set(want)
    bad = [k for k in want if got[k] != want[k]]
    assert not bad, f"oracle differs from the reference on {bad}"


def test_oracle_kats(oracle):
    g = golden("kat.json")
    hw = HostWeights.bind_test_kat()
    assert list(oracle.generate(hw.desc, [1, 2, 3], 3, max_seq=8)) == g["bind_123"]
    assert list(oracle.generate(hw.desc, [5, 6, 7], 3, max_seq=8)) == g["bind_567"]
    hs = HostWeights.shift_demo_kat()
    assert list(oracle.generate(hs.desc, list(range(97, 105)), 16, max_seq=1024)) == g["shift_abcdefgh"]


def test_oracle_c0_greedy_and_logits(oracle):
    g = golden("c0.json")
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic(cfg)
    pr = prompt_ids(cfg)
    assert list(pr) == g["prompt"]
    assert list(oracle.generate(hw.desc, pr, cfg.new_tokens, max_seq=cfg.max_seq)) == g["greedy"]
    rows, kv = make_golden.teacher_forced(oracle, hw, pr, 16)
    assert [r["sha"] for r in rows] == [r["sha"] for r in g["teacher_forced"]]
    assert kv == g["kv_sha"]


def test_oracle_sampler_and_penalty_match_reference(oracle):
    """jyo_sample (the generate.h:50-77 restatement) reproduces the reference's
    sampled (T 0.8) and repetition-penalised (1.3) sequences on configs[0]."""
    g = golden("c0.json")
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic(cfg)
    pr = prompt_ids(cfg)
    got = oracle.generate(hw.desc, pr, 64, temperature=0.8, rep=1.3, max_seq=cfg.max_seq)
    assert list(got) == g["sampled_t0.8_p1.3"]
    got = oracle.generate(hw.desc, pr, 64, temperature=0.0, rep=1.3, max_seq=cfg.max_seq)
    assert list(got) == g["greedy_p1.3"]


def test_oracle_c1_shape(oracle):
    g = golden("c1.json")
    cfg = CONFIGS["c1"]
    hw = HostWeights.synthetic(cfg)
    pr = prompt_ids(cfg, n=16)
    assert list(pr) == g["prompt"]
    assert list(oracle.generate(hw.desc, pr, 16, max_seq=cfg.max_seq)) == g["greedy"]
    rows, kv = make_golden.teacher_forced(oracle, hw, pr, 4)
    assert [r["sha"] for r in rows] == [r["sha"] for r in g["teacher_forced"]]
    assert kv == g["kv_sha"]


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__))), "oracle", "_ref", "libjyref.so")), reason="reference build absent")
def test_reference_build_still_matches_golden():
    """The prebuilt reference harness (oracle/_ref) reproduces the fixtures on this host."""
    from oracle.bind import Reference
    ref = Reference("fma", 0)
    want = golden("ops.json")["ops"]
    got = make_golden.run_ops(ref)
    assert got == want


@pytest.mark.parametrize("name", ["c2_4096_2l", "c2_16384_2l"])
def test_oracle_long_context_matches_reference(oracle, name):
    """Teacher-forced steps from a seeded 4096- / 16384-position int8 K/V
    context (tests/golden/longctx.json, the reference's own fma path): the
    oracle's logits are bit-identical at every step."""
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden_longctx as mgl
    case = golden("longctx.json")[name]
    hw = HostWeights.synthetic(mgl.long_cfg(case["config"], case["ctx"], case["layers"]))
    out, fed = mgl.run(oracle, hw, case["ctx"], None)
    assert fed == case["fed"]
    assert [sha(x) for x in out] == [r["sha"] for r in case["steps"]]


def test_oracle_f16_matches_reference(oracle):
    """fp16 weights (matmul_f16.h:19-41 through matmul_w; tests/golden/f16.json,
    the reference's own fma path): the oracle's matmul_f16 digests, tail
    columns included, and the greedy sequence of the configs[0] shape with
    fp16 linear matrices, LM head and embedding are identical."""
    import make_golden_f16 as mgf
    g = golden("f16.json")
    for m, n, k in mgf.F16_CASES:
        a, b = mgf.f16_inputs(m, n, k)
        c = np.empty(m * n, np.float32)
        oracle.matmul_f16(ptr(a), ptr(b), ptr(c), m, n, k)
        assert sha(c) == g["ops"][f"f16_{m}_{n}_{k}"], (m, n, k)
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic_f16(cfg)
    pr = prompt_ids(cfg)
    assert list(pr) == g["c0_f16"]["prompt"]
    assert list(oracle.generate(hw.desc, pr, 64, max_seq=cfg.max_seq)) == g["c0_f16"]["greedy"]
