"""The reference's operator and generate entry points through
include/jieyu_b200_shim.hpp (called exactly as the reference's code calls its
own: host pointers, the reference's structs, synchronous) against the CPU
oracle on seeded inputs. Tolerances are those of the device entry points
underneath (tests/test_gpu_ops.py): the shim only moves the operands."""
import ctypes as C

import numpy as np
import pytest

import _shim
from _kquant import kquant_blocks
from _util import f32, golden, ptr
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, HostWeights, prompt_ids, rope_table, synth_f32, synth_q8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def shim(cuda, tmp_path_factory):
    lib = _shim.build(str(tmp_path_factory.mktemp("shim")))
    yield lib
    lib.shim_release()


def _ok(lib, r):
    assert r >= 0, lib.shim_last_error().decode()
    return r


@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (5, 96, 1024), (24, 128, 2048)])
def test_matmul_q_q8_0(shim, oracle, m, n, k):
    w = synth_q8(21, n + k, n, k)
    a = synth_f32(22, m + k, m * k, 1.0)
    want = np.empty(m * n, np.float32)
    oracle.matmul_q8(ptr(a), ptr(w), ptr(want), m, n, k)
    got = np.empty_like(want)
    _ok(shim, shim.shim_matmul_q(ptr(a), ptr(w), ptr(got), m, n, k, _capi.JYC_Q8_0))
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


@pytest.mark.parametrize("qt", [_capi.JYC_Q4K, _capi.JYC_Q5K, _capi.JYC_Q6K])
def test_matmul_q_kquant(shim, oracle, qt):
    m, n, k = 3, 64, 512
    w = kquant_blocks(qt, n, k, seed=5)
    a = synth_f32(23, k, m * k, 1.0)
    want = np.empty(m * n, np.float32)
    oracle.matmul_qk(ptr(a), ptr(w), ptr(want), m, n, k, qt)
    got = np.empty_like(want)
    _ok(shim, shim.shim_matmul_q(ptr(a), ptr(w), ptr(got), m, n, k, qt))
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


def test_matmul_and_matmul_w(shim, oracle):
    m, n, k = 4, 96, 160
    A = synth_f32(24, 1, m * k, 1.0)
    B = synth_f32(25, 2, k * n, 0.05)  # [k][n]
    want = np.empty(m * n, np.float32)
    oracle.matmul_f32(m, n, k, ptr(A), ptr(B), ptr(want))
    got = np.empty_like(want)
    _ok(shim, shim.shim_matmul(m, n, k, ptr(A), ptr(B), ptr(got)))
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()
    got_w = np.empty_like(want)
    _ok(shim, shim.shim_matmul_w(ptr(B), None, 0, m, n, k, ptr(A), ptr(got_w)))
    assert np.array_equal(got_w, got)
    # Q8_0 WMat: the same as matmul_q; an empty WMat: C = 0 (wmat_kernel.h:12-13)
    wq = synth_q8(26, 3, n, k)
    _ok(shim, shim.shim_matmul_w(None, ptr(wq), _capi.JYC_Q8_0, m, n, k, ptr(A), ptr(got_w)))
    oracle.matmul_q8(ptr(A), ptr(wq), ptr(want), m, n, k)
    assert np.abs(got_w - want).max() <= 2e-5 * np.abs(want).max()
    _ok(shim, shim.shim_matmul_w(None, None, 0, m, n, k, ptr(A), ptr(got_w)))
    assert not got_w.any()


def test_rmsnorm_rope_silu_kvpack(shim, oracle):
    n = 2048
    x = synth_f32(27, 1, n, 1.0)
    w = synth_f32(28, 1, n, 1.0) + np.float32(1.0)
    want, got = np.empty_like(x), np.empty_like(x)
    oracle.rmsnorm(ptr(x), ptr(want), ptr(w), n, f32(1e-5))
    _ok(shim, shim.shim_rmsnorm(ptr(x), ptr(got), ptr(w), n, 1e-5))
    assert np.abs(got - want).max() <= 4e-7 * np.abs(want).max()
    # RoPE in place at start_pos 40 (bit-exact)
    hd, heads, seq, start = 64, 6, 5, 40
    cos, sin = rope_table(96, hd, 5e5)
    q = synth_f32(29, 1, seq * heads * hd, 1.0)
    qo, qs = q.copy(), q.copy()
    oracle.rope_pos(ptr(qo), seq, start, heads, hd, ptr(cos), ptr(sin))
    _ok(shim, shim.shim_rope_pos(ptr(qs), seq, start, heads, hd, ptr(cos), ptr(sin)))
    assert np.array_equal(qs, qo)
    # silu (the reference's own exp polynomial: bit-exact)
    s_want, s_got = np.empty_like(x), np.empty_like(x)
    oracle.silu(ptr(x), ptr(s_want), n)
    _ok(shim, shim.shim_silu(ptr(x), ptr(s_got), n))
    assert np.array_equal(s_got, s_want)
    # kv_pack_q8 (bit-exact)
    rows, kvh = 3, 4
    src = synth_f32(30, 1, rows * kvh * hd, 1.0)
    d0, d1 = np.empty(src.size, np.int8), np.empty(src.size, np.int8)
    c0, c1 = np.empty(rows * kvh, np.float32), np.empty(rows * kvh, np.float32)
    oracle.kv_pack_q8(ptr(src), ptr(d0), ptr(c0), kvh, hd, rows)
    _ok(shim, shim.shim_kv_pack_q8(ptr(src), ptr(d1), ptr(c1), kvh, hd, rows))
    assert np.array_equal(d0, d1) and np.array_equal(c0, c1)


@pytest.mark.parametrize("seq,start", [(1, 0), (3, 40), (1, 700)])
def test_attention_q8_with_the_callers_cache(shim, oracle, seq, start):
    H, KV, hd, cap = 32, 8, 64, 768
    qd, kvd = H * hd, KV * hd
    rng = np.random.default_rng(seq * 1000 + start)
    ctx = {}
    for name in ("k", "v"):
        ctx[name] = rng.integers(-127, 128, size=cap * kvd, dtype=np.int8)
        ctx[name + "s"] = (rng.uniform(0.2, 0.5, size=cap * KV) / 127).astype(np.float32)
    Q = synth_f32(31, seq, seq * qd, 1.0)
    K = synth_f32(32, seq, seq * kvd, 1.0)
    V = synth_f32(33, seq, seq * kvd, 1.0)
    caches = [{k: v.copy() for k, v in ctx.items()} for _ in range(2)]
    outs = [np.empty(seq * qd, np.float32) for _ in range(2)]
    c = caches[0]
    assert oracle.attention_q8(ptr(Q), ptr(K), ptr(V), ptr(outs[0]), seq, start, H, KV, hd, ptr(c["k"]),
                               ptr(c["ks"]), ptr(c["v"]), ptr(c["vs"]), cap) == 0
    c = caches[1]
    _ok(shim, shim.shim_attention_q8(ptr(Q), ptr(K), ptr(V), ptr(outs[1]), seq, start, H, KV, hd, ptr(c["k"]),
                                     ptr(c["ks"]), ptr(c["v"]), ptr(c["vs"]), cap))
    assert np.abs(outs[1] - outs[0]).max() <= 1e-5 * np.abs(outs[0]).max()
    for name in ("k", "v", "ks", "vs"):  # appended rows bit-exact, the rest untouched
        assert np.array_equal(caches[1][name], caches[0][name]), name


def test_attention_q8_without_a_cache(shim, oracle):
    """An incomplete __KVq: a temporary cache of seq rows at position 0 (attention_q8.h:40-46)."""
    H, KV, hd, seq = 8, 4, 64, 5
    Q = synth_f32(34, 1, seq * H * hd, 1.0)
    K = synth_f32(35, 1, seq * KV * hd, 1.0)
    V = synth_f32(36, 1, seq * KV * hd, 1.0)
    want, got = np.empty(seq * H * hd, np.float32), np.empty(seq * H * hd, np.float32)
    tk, tv = np.empty(seq * KV * hd, np.int8), np.empty(seq * KV * hd, np.int8)
    ts, tvs = np.empty(seq * KV, np.float32), np.empty(seq * KV, np.float32)
    assert oracle.attention_q8(ptr(Q), ptr(K), ptr(V), ptr(want), seq, 0, H, KV, hd, ptr(tk), ptr(ts), ptr(tv),
                               ptr(tvs), seq) == 0
    _ok(shim, shim.shim_attention_q8(ptr(Q), ptr(K), ptr(V), ptr(got), seq, 9, H, KV, hd, None, None, None, None, 0))
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


def test_ffn(shim, oracle):
    seq, D, F = 2, 512, 1376
    x = synth_f32(37, 1, seq * D, 1.0)
    ws = [synth_q8(38, i, F if i != 1 else D, D if i != 1 else F) for i in range(3)]  # w1 [F][D], w2 [D][F], w3
    g, u = np.empty(seq * F, np.float32), np.empty(seq * F, np.float32)
    oracle.matmul_q8(ptr(x), ptr(ws[0]), ptr(g), seq, F, D)
    oracle.matmul_q8(ptr(x), ptr(ws[2]), ptr(u), seq, F, D)
    oracle.silu(ptr(g), ptr(g), seq * F)
    h = (g * u).astype(np.float32)
    want = np.empty(seq * D, np.float32)
    oracle.matmul_q8(ptr(h), ptr(ws[1]), ptr(want), seq, D, F)
    wm = [_capi.WMat() for _ in range(3)]
    for i in range(3):
        wm[i].q = ptr(ws[i])
        wm[i].qt = _capi.JYC_Q8_0
    got = np.empty_like(want)
    _ok(shim, shim.shim_ffn(ptr(x), C.byref(wm[0]), C.byref(wm[1]), C.byref(wm[2]), ptr(got), seq, D, F))
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_generate_configs0_greedy(shim):
    """generate() with the reference's argument list on configs[0]: the
    reference's own 128-token greedy sequence (tests/golden/c0.json); a
    token callback that stops after 3 tokens; a second call reuses the bound
    model."""
    g = golden("c0.json")
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic(cfg)
    pr = np.array(g["prompt"], np.int32)
    out = np.zeros(cfg.max_seq + 1, np.int32)
    n = _ok(shim, shim.shim_generate(C.byref(hw.desc), ptr(pr), len(pr), None, 0, 128, 0.0, 1.0, 0, ptr(out)))
    assert n == 160 and list(out[:n]) == g["greedy"]
    n = _ok(shim, shim.shim_generate(C.byref(hw.desc), ptr(pr), len(pr), None, 0, 128, 0.0, 1.0, 3, ptr(out)))
    assert n == 35 and list(out[:n]) == g["greedy"][:35]
    # sampling and the repetition penalty: the reference's sequences
    n = _ok(shim, shim.shim_generate(C.byref(hw.desc), ptr(pr), len(pr), None, 0, 64, 0.0, 1.3, 0, ptr(out)))
    assert list(out[:n]) == g["greedy_p1.3"]


def test_generate_cached_fills_the_callers_cache(shim, oracle):
    cfg = CONFIGS["c0"]
    hw = HostWeights.synthetic(cfg)
    pr = prompt_ids(cfg)
    out = np.zeros(cfg.max_seq + 1, np.int32)
    k = np.empty(cfg.max_seq * cfg.kv_dim, np.int8)
    v = np.empty_like(k)
    ks = np.empty(cfg.max_seq * cfg.kv_heads, np.float32)
    vs = np.empty_like(ks)
    cur = C.c_int(-1)
    n = _ok(shim, shim.shim_generate_cached(C.byref(hw.desc), ptr(pr), len(pr), 8, ptr(out), 0, ptr(k), ptr(ks),
                                            ptr(v), ptr(vs), C.byref(cur)))
    want = oracle.generate(hw.desc, pr, 8, max_seq=cfg.max_seq)
    assert n == len(want) and list(out[:n]) == list(want)
    assert cur.value == n - 1  # every position but the last new token went through forward_cached
    # layer 0 sees identical inputs: its cache rows equal the oracle's (fed
    # the same way: the prompt in one forward, then one token per step)
    cache = oracle.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    try:
        logits = np.empty(cfg.vocab, np.float32)
        P = len(pr)
        ids = np.ascontiguousarray(out[:P], np.int32)
        assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(ids), P, 0, ptr(logits), None) == 0
        for pos in range(P, n - 1):
            t = np.ascontiguousarray(out[pos:pos + 1], np.int32)
            assert oracle.forward_logits(C.byref(hw.desc), cache, ptr(t), 1, pos, ptr(logits), None) == 0
        ok, oks, ov, ovs = (np.empty_like(a[: cur.value * (a.size // cfg.max_seq)]) for a in (k, ks, v, vs))
        oracle.cache_read(cache, 0, cur.value, ptr(ok), ptr(oks), ptr(ov), ptr(ovs))
        nk = cur.value * cfg.kv_dim
        assert np.array_equal(k[:nk], ok) and np.array_equal(v[:nk], ov)
    finally:
        oracle.cache_free(cache)
