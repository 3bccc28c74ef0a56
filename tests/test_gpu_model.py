"""Model-level parity of the device token loop (jyc_model_create / jyc_generate
/ jyc_forward_logits) against the reference: golden fixtures produced by the
reference itself (tests/golden) and the bit-identical CPU oracle.

Bars (north star): greedy token ids identical; logits within
LOGIT_TOL * max|logit|; argmax equal wherever the reference's top-2 gap
exceeds twice the tolerance (near ties are reported, not failed).

The reference is not self-consistent to that bar on every shape: its own
scalar and fma code paths, on identical inputs, differ by 0.9e-3
to 2.2-3.8e-3 of max|logit|, and their int8 KV
bytes at the last layer by 3-12 % (fp32 rounding differences amplified
through the layers). The fixtures record that spread (tests/golden,
isa_spread); the logit tolerance is max(LOGIT_TOL, 1.5 x the largest spread)
and the last-layer KV byte mismatch may reach max(1e-3, 1.5 x the
reference's own fraction). Layer 0 (identical inputs) stays bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

from _util import LOGIT_TOL, golden, ptr
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c0(cuda):
    hw = HostWeights.synthetic(CONFIGS["c0"])
    m = DeviceModel(hw)
    yield hw, m
    m.close()


def test_kat_bind_weights(cuda):
    """check_bind_weights cases 6 and 9 (libs/text/text.h:817-913)."""
    g = golden("kat.json")
    m = DeviceModel(HostWeights.bind_test_kat())
    assert list(m.generate(np.array([1, 2, 3]), 3)) == g["bind_123"]
    a = m.generate(np.array([5, 6, 7]), 3)
    b = m.generate(np.array([5, 6, 7]), 3)
    assert list(a) == g["bind_567"] and list(a) == list(b)
    m.close()


def test_kat_shift_demo(cuda):
    """check_pipeline case 6 (libs/text/text.h:993-1002): "abcdefgh" -> "ijklmnopqrstuvwx"."""
    g = golden("kat.json")
    m = DeviceModel(HostWeights.shift_demo_kat())
    out = m.generate(np.arange(97, 105), 16)
    assert list(out) == g["shift_abcdefgh"]
    assert bytes(out[8:].astype(np.uint8)).decode() == "ijklmnopqrstuvwx"
    m.close()


def test_q8_models_decode_with_the_megakernel(c0):
    hw, m = c0
    lib = _capi.load()
    assert lib.jyc_model_decode_path(m.h) == 2
    assert lib.jyc_model_kernels_per_step(m.h) == 1
    assert lib.jyc_device_error(0) == 0


def test_c0_greedy_128_tokens_identical(c0):
    """32-token prompt, 128 greedy tokens == the reference's."""
    hw, m = c0
    g = golden("c0.json")
    prompt = np.array(g["prompt"], dtype=np.int32)
    assert list(prompt) == list(prompt_ids(hw.cfg))
    out = m.generate(prompt, hw.cfg.new_tokens)
    assert len(out) == len(g["greedy"]) == 32 + 128
    assert list(out) == g["greedy"]


def _teacher_forced(m, hw, oracle, prompt, steps):
    """Device and oracle fed the same tokens; yields (step, device, oracle) logits."""
    cfg = hw.cfg
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    want = np.empty(cfg.vocab, np.float32)
    tok = np.ascontiguousarray(prompt, np.int32)
    pos = 0
    try:
        for s in range(steps + 1):
            got = m.forward_logits(tok, pos)
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(tok), len(tok), pos,
                                         ptr(want), None) == 0
            yield s, got, want.copy(), cache, pos + len(tok)
            pos += len(tok)
            tok = np.array([int(np.argmax(want))], np.int32)
    finally:
        oracle.cache_free(cache)


def _tol(spread, step):
    """Logit tolerance: max(LOGIT_TOL, 1.5 x the reference's own scalar-vs-fma
    spread, the largest over the fixture's steps: the amplification is a
    property of the model, the per-step value a sample of it)."""
    if spread is None:
        return LOGIT_TOL
    return max(LOGIT_TOL, 1.5 * max(spread["logits_rel"]))


def _check_logits(got, want, ref_row=None, tol=LOGIT_TOL, label=""):
    amax = np.abs(want).max()
    err = np.abs(got - want).max()
    print(f"  {label} max|dlogit|/max|logit| = {err / amax:.2e} (bar {tol:.2e})")
    assert err <= tol * amax, f"max|dlogit| {err} > {tol} * {amax}"
    top = np.sort(want.astype(np.float64))[-2:]
    gap = top[1] - top[0]
    if gap > 2 * tol * amax:
        assert int(np.argmax(got)) == int(np.argmax(want))
    if ref_row is not None:
        assert int(np.argmax(want)) == ref_row["argmax"]
    return err / amax


def test_c0_teacher_forced_logits(c0, oracle):
    hw, m = c0
    g = golden("c0.json")
    rels = []
    for s, got, want, cache, n in _teacher_forced(m, hw, oracle, g["prompt"], 16):
        rels.append(_check_logits(got, want, g["teacher_forced"][s], _tol(g["isa_spread"], s), f"c0 step {s}"))
    assert max(rels) < LOGIT_TOL  # configs[0] meets the 1e-3 bar outright


def test_c0_kv_cache_bytes(c0, oracle):
    """int8 KV rows the device appended vs the oracle's: layer 0 (identical
    inputs) bit-exact; deeper layers differ by at most one quantisation step,
    on no more entries than the reference's own two code paths disagree on."""
    hw, m = c0
    cfg = hw.cfg
    g = golden("c0.json")
    last = None
    for s, got, want, cache, n in _teacher_forced(m, hw, oracle, g["prompt"], 3):
        last = (cache, n)
        if s == 3:
            cache, n = last
            for layer in (0, cfg.layers - 1):
                k = np.empty(n * cfg.kv_dim, np.int8)
                v = np.empty_like(k)
                ks = np.empty(n * cfg.kv_heads, np.float32)
                vs = np.empty_like(ks)
                oracle.cache_read(cache, layer, n, ptr(k), ptr(ks), ptr(v), ptr(vs))
                dk, dks, dv, dvs = m.read_kv(layer, n)
                frac = max(1e-3, 1.5 * g["isa_spread"]["kv_frac"][str(layer)])
                for a, b in ((dk, k), (dv, v)):
                    diff = np.abs(a.astype(np.int32) - b.astype(np.int32))
                    assert diff.max() <= 1 and (diff > 0).mean() <= frac
                rtol = 1e-5 if layer == 0 else 2e-3
                for a, b in ((dks, ks), (dvs, vs)):
                    assert np.allclose(a, b, rtol=rtol, atol=0)
                if layer == 0:
                    # layer 0 sees identical inputs (embedding rows): bit-exact
                    assert np.array_equal(dk, k) and np.array_equal(dv, v)


def test_c1_shape_greedy_and_logits(cuda, oracle):
    """configs[1] shape (tied Q8_0 embedding, QKV bias, theta 1e6)."""
    g = golden("c1.json")
    hw = HostWeights.synthetic(CONFIGS["c1"])
    m = DeviceModel(hw)
    out = m.generate(np.array(g["prompt"], np.int32), 16)
    assert list(out) == g["greedy"]
    for s, got, want, cache, n in _teacher_forced(m, hw, oracle, g["prompt"], 4):
        _check_logits(got, want, g["teacher_forced"][s], _tol(g["isa_spread"], s), f"c1 step {s}")
    m.close()


@pytest.mark.parametrize("key", ["c2", "c2f"])
def test_c2_shapes_short(cuda, oracle, key):
    """configs[2] shape, Q8_0 and fp32 variants: 8-token prompt + 3 steps."""
    from dataclasses import replace
    cfg = replace(CONFIGS[key], max_seq=256)
    hw = HostWeights.synthetic(cfg)
    m = DeviceModel(hw)
    pr = prompt_ids(cfg, n=8)
    spread = golden("c2.json")[key]["isa_spread"]
    for s, got, want, cache, n in _teacher_forced(m, hw, oracle, pr, 3):
        _check_logits(got, want, tol=_tol(spread, s), label=f"{key} step {s}")
    m.close()


@pytest.mark.parametrize("key", ["c1", "c2"])
def test_decode_kernel_step_from_the_oracle_state(cuda, oracle, key):
    """One decode-kernel step at a time against the north-star bar
    (max|dlogit| <= 1e-3 max|logit|, no allowance for the reference's own
    spread): before every step the oracle's whole int8 KV cache (its prefill
    of a 16-token prompt, then its own steps; the reference's code paths) is
    copied into the device's (jyc_model_write_kv), so each step starts from
    the reference's state. The prompt-based tests above differ from the
    oracle by 1-4e-3: two prefills that round differently, and then steps
    that append their own KV rows, drift apart through the int8 KV
    quantisation as the reference's scalar and fma paths do. With the state
    shared, one step's error comes only from the int8 rounding steps that a
    last-bit difference in fp32 (summation order, the 21-bit activation
    digits) flips inside that step: configs[1] stays below 1e-4 on every
    step; configs[2] (16 layers of 2048) mostly below 5e-4 with an
    occasional step just above 1e-3. The bar: the median step inside 1e-3,
    every step inside the reference's own scalar-vs-fma spread allowance.
    The free-running error of the same steps is printed for comparison."""
    from dataclasses import replace
    cfg = CONFIGS[key] if key == "c1" else replace(CONFIGS[key], max_seq=256)
    hw = HostWeights.synthetic(cfg)
    m = DeviceModel(hw)
    P, steps = 16, 8
    spread = golden("c1.json")["isa_spread"] if key == "c1" else golden("c2.json")[key]["isa_spread"]
    spread_tol = _tol(spread, 0)
    pr = np.ascontiguousarray(prompt_ids(cfg, n=P), np.int32)
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    want = np.empty(cfg.vocab, np.float32)
    try:
        assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(pr), P, 0, ptr(want), None) == 0
        toks = []
        errs = []
        for s in range(steps):
            n = P + s
            k = np.empty(n * cfg.kv_dim, np.int8)
            v = np.empty_like(k)
            ks = np.empty(n * cfg.kv_heads, np.float32)
            vs = np.empty_like(ks)
            for layer in range(cfg.layers):
                oracle.cache_read(cache, layer, n, ptr(k), ptr(ks), ptr(v), ptr(vs))
                m.write_kv(layer, k, ks, v, vs)
            tok = int(np.argmax(want))
            toks.append(tok)
            t = np.array([tok], np.int32)
            got = m.forward_logits(t, n)
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(t), 1, n, ptr(want), None) == 0
            errs.append(_check_logits(got, want, tol=spread_tol, label=f"{key} step {s} from the oracle's state"))
        # the same steps free-running from the shared prefill (printed only)
        k = np.empty(P * cfg.kv_dim, np.int8)
        v = np.empty_like(k)
        ks = np.empty(P * cfg.kv_heads, np.float32)
        vs = np.empty_like(ks)
        ocache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
        try:
            assert oracle.forward_logits(C.byref(hw.desc), ocache, ptr(pr), P, 0, ptr(want), None) == 0
            for layer in range(cfg.layers):
                oracle.cache_read(ocache, layer, P, ptr(k), ptr(ks), ptr(v), ptr(vs))
                m.write_kv(layer, k, ks, v, vs)
            for s, tok in enumerate(toks):
                t = np.array([tok], np.int32)
                got = m.forward_logits(t, P + s)
                assert oracle.forward_logits(C.byref(hw.desc), ocache, ptr(t), 1, P + s, ptr(want), None) == 0
                print(f"  {key} step {s} free-running: max|dlogit|/max|logit| = "
                      f"{np.abs(got - want).max() / np.abs(want).max():.2e}")
        finally:
            oracle.cache_free(ocache)
        assert float(np.median(errs)) < LOGIT_TOL
        if key == "c1":
            assert max(errs) < LOGIT_TOL
    finally:
        oracle.cache_free(cache)
        m.close()


def test_prefill_in_several_passes(cuda, oracle, monkeypatch):
    """A prompt longer than one prefill pass (JYC_PF_ROWS=64: a 256-token
    prompt in 4 passes, each pass attending over the cache rows the earlier
    ones wrote) gives the logits of one pass within the model tolerance, and
    both stay within it of the oracle."""
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic(cfg)
    pr = np.ascontiguousarray(prompt_ids(cfg, n=256), np.int32)
    want = np.empty(cfg.vocab, np.float32)
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    try:
        assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(pr), len(pr), 0, ptr(want), None) == 0
    finally:
        oracle.cache_free(cache)
    got = {}
    for rows in ("64", None):
        if rows:
            monkeypatch.setenv("JYC_PF_ROWS", rows)
        else:
            monkeypatch.delenv("JYC_PF_ROWS", raising=False)
        m = DeviceModel(hw)
        got[rows] = m.forward_logits(pr, 0)
        m.close()
    tol = _tol(golden("c0.json")["isa_spread"], 0)
    for rows, g in got.items():
        _check_logits(g, want, tol=tol, label=f"c0 prompt of 256 in passes of {rows or 'one'}")
    amax = np.abs(want).max()
    assert np.abs(got["64"] - got[None]).max() <= tol * amax


def test_generate_contract_edges(c0):
    hw, m = c0
    pr = prompt_ids(hw.cfg)
    lib = _capi.load()
    out = np.zeros(hw.cfg.max_seq + 1, np.int32)
    e = np.zeros(1, np.int32)
    cb = _capi.TOKEN_CB()
    # prompt_len <= 0 or > max_seq -> 0 (generate.h:25)
    assert lib.jyc_generate(m.h, ptr(pr), 0, ptr(e), 0, 4, 0.0, ptr(out), 1.0, cb, None) == 0
    big = np.zeros(hw.cfg.max_seq + 1, np.int32)
    assert lib.jyc_generate(m.h, ptr(big), len(big), ptr(e), 0, 4, 0.0, ptr(out), 1.0, cb, None) == 0
    # max_new <= 0 -> prompt_len (generate.h:32)
    assert lib.jyc_generate(m.h, ptr(pr), 32, ptr(e), 0, 0, 0.0, ptr(out), 1.0, cb, None) == 32
    # prompt fills the context: nothing generated
    full = prompt_ids(hw.cfg, n=hw.cfg.max_seq)
    assert len(m.generate(full, 4)) == hw.cfg.max_seq
    # context limit: len stops at max_seq
    near = prompt_ids(hw.cfg, n=hw.cfg.max_seq - 3)
    assert len(m.generate(near, 50)) == hw.cfg.max_seq
    # out-of-range id -> error
    bad = pr.copy()
    bad[3] = hw.cfg.vocab
    with pytest.raises(_capi.JycError):
        m.generate(bad, 2)


def test_generate_eos_and_callback(c0):
    hw, m = c0
    g = golden("c0.json")
    pr = np.array(g["prompt"], np.int32)
    ref = g["greedy"]
    # EOS = the 5th generated token: generation stops right after emitting it
    eos_tok = ref[32 + 4]
    first = ref[32:].index(eos_tok)
    out = m.generate(pr, 100, eos=[eos_tok])
    assert list(out) == ref[: 32 + first + 1]
    # callback asks to stop after 3 tokens (generate.h:79)
    seen = []
    out = m.generate(pr, 100, cb=lambda t: (seen.append(t), len(seen) >= 3)[1])
    assert seen == ref[32:35] and list(out) == ref[:35]


def _forced_rows(m, hw, oracle, ids, P):
    """Device and oracle fed the same sequence `ids` (prompt = ids[:P]); yields
    (step, device logits, oracle logits) for the pick of ids[P + step]."""
    cfg = hw.cfg
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    want = np.empty(cfg.vocab, np.float32)
    try:
        pos = 0
        for s in range(len(ids) - P):
            tok = np.ascontiguousarray(ids[:P] if s == 0 else ids[P + s - 1:P + s], np.int32)
            got = m.forward_logits(tok, pos)
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(tok), len(tok), pos, ptr(want), None) == 0
            yield s, got, want.copy()
            pos += len(tok)
    finally:
        oracle.cache_free(cache)


def _replay_picks(m, hw, oracle, ids, P, T, pen, tol):
    """Checks a device-generated sequence step by step. At every step the
    reference's pick (jyo_sample, generate.h:50-77) from the DEVICE's logits
    must be the device's token (the sampler exact), and the pick from the
    ORACLE's logits (the reference's own) may differ only where the draw lies
    within what the logit difference (itself within `tol`) can move across a
    bucket boundary: |r - cdf_k| / sum <= exp(4 max|dlogit| / T) - 1 (greedy:
    a top-2 gap within 2 max|dlogit|; dlogit after the penalty). Returns the
    steps where they differ."""
    V = hw.cfg.vocab
    ids = np.ascontiguousarray(ids, np.int32)
    rng_d, rng_o = C.c_uint(12345), C.c_uint(12345)
    flips = []
    for s, dl, ol in _forced_rows(m, hw, oracle, ids, P):
        _check_logits(dl, ol, tol=tol)
        pen_rows = []
        for row in (dl, ol):  # the penalised rows (T 0: jyo_sample stops after the penalty and an argmax)
            row = row.copy()
            oracle.lib.jyo_sample(ptr(row), V, 0.0, pen, ptr(ids), P, P + s, C.byref(C.c_uint(0)))
            pen_rows.append(row.astype(np.float64))
        delta = float(np.abs(pen_rows[0] - pen_rows[1]).max())
        dl, ol = dl.copy(), ol.copy()
        pd = oracle.lib.jyo_sample(ptr(dl), V, T, pen, ptr(ids), P, P + s, C.byref(rng_d))
        po = oracle.lib.jyo_sample(ptr(ol), V, T, pen, ptr(ids), P, P + s, C.byref(rng_o))
        assert pd == ids[P + s], f"step {s}: device token {ids[P + s]} != sampler on its logits {pd}"
        if po == pd:
            continue
        if T > 0:
            c = np.cumsum(ol.astype(np.float64))  # the probabilities jyo_sample wrote back
            r = (rng_o.value >> 8) / 16777216.0 * c[-1]
            margin = abs(r - c[min(po, pd)]) / c[-1]
            assert margin <= np.expm1(4 * delta / T), f"step {s}: draw {margin:.3g} from the boundary"
        else:
            assert abs(float(ol[po]) - float(ol[pd])) <= 2 * delta, f"step {s}: not a near tie"
        flips.append(s)
    return flips


@pytest.mark.parametrize("T,pen,key", [(0.8, 1.3, "sampled_t0.8_p1.3"), (0.0, 1.3, "greedy_p1.3")])
def test_c0_sampled_and_penalised_match_reference(c0, oracle, T, pen, key):
    """configs[0], 64 new tokens sampled at T 0.8 / greedy, repetition penalty
    1.3 (the decode kernel samples in its head phase; the prefill's first
    token is re-picked by the sampler kernel). The device's sequence equals
    the reference's up to the first step where the two logits rows (equal
    within the logit tolerance) fall on either side of the draw; every step
    is replayed (`_replay_picks`), at most 2 such steps in 64."""
    hw, m = c0
    g = golden("c0.json")
    spread = g.get("isa_spread")
    pr = np.array(g["prompt"], np.int32)
    P = len(pr)
    got = m.generate(pr, 64, temperature=T, repetition_penalty=pen)
    ref = g[key]
    assert len(got) == len(ref) == P + 64
    flips = _replay_picks(m, hw, oracle, got, P, T, pen, _tol(spread, 0))
    assert len(flips) <= 2, flips
    first = flips[0] if flips else 64
    assert list(got[:P + first]) == ref[:P + first]
    # a later greedy call is unaffected (the sampler state resets per call)
    assert list(m.generate(pr, 8)) == g["greedy"][: P + 8]


def test_sampling_on_the_per_op_path_matches_oracle(cuda, oracle):
    """The f32 bind-weights model decodes through the per-op step (no decode
    kernel; the sampler kernel re-picks every head's token): each sequence is
    replayed against the oracle (`_replay_picks`) and equals the oracle's own
    up to the first boundary flip (none expected); with a callback (block-wise
    stepping) the device gives the same sequence."""
    hw = HostWeights.bind_test_kat()
    m = DeviceModel(hw)
    lib = _capi.load()
    assert lib.jyc_model_decode_path(m.h) != 2
    pr = np.array([1, 2, 3], np.int32)
    for T, pen in ((0.8, 1.3), (1.5, 1.0), (0.0, 1.3)):
        got = m.generate(pr, 12, temperature=T, repetition_penalty=pen)
        assert len(got) == hw.cfg.max_seq
        flips = _replay_picks(m, hw, oracle, got, 3, T, pen, LOGIT_TOL)
        first = flips[0] if flips else len(got) - 3
        want = oracle.generate(hw.desc, pr, 12, temperature=T, rep=pen, max_seq=hw.cfg.max_seq)
        assert list(got[:3 + first]) == list(want[:3 + first])
        seen = []
        again = m.generate(pr, 12, temperature=T, repetition_penalty=pen, cb=lambda t: (seen.append(t), False)[1])
        assert list(again) == list(got) and seen == list(got[3:])
    m.close()
