"""Operator parity: each CUDA entry point of libjieyu_b200.so against the CPU
oracle (which is bit-identical to the reference) on the same seeded inputs.

Bit-exact where the reference's arithmetic is order-free (int8 quantisation,
KV bytes, RoPE, SiLU vector body, argmax); otherwise the tolerance is stated
next to each comparison.
"""
import ctypes as C

import numpy as np
import pytest

from _util import dev, f32, host, libc_rand_fill, ptr, stream
from jieyu_b200 import _capi
from jieyu_b200.model import CONFIGS, rope_table, synth_f32, synth_q8

pytestmark = pytest.mark.gpu


def _lib():
    return _capi.load()


def _q8_dev(torch, blocks: np.ndarray, n: int, k: int):
    lib = _lib()
    b = dev(torch, blocks)
    qs = torch.empty(n * k, dtype=torch.uint8, device="cuda")
    d = torch.empty(n * (k // 32), dtype=torch.int16, device="cuda")
    _capi.check(lib.jyc_q8_repack(b.data_ptr(), n, k, qs.data_ptr(), d.data_ptr(), stream(torch)))
    return qs, d


def _gemv_shapes():
    shapes = set()
    for key in ("c0", "c1", "c2", "c3"):
        c = CONFIGS[key]
        D, F = c.hidden, c.inter
        for nk in ((c.q_dim, D), (c.kv_dim, D), (D, c.q_dim), (F, D), (D, F)):
            shapes.add(nk)
    shapes.add((CONFIGS["c0"].vocab, CONFIGS["c0"].hidden))
    shapes.add((CONFIGS["c1"].vocab, CONFIGS["c1"].hidden))
    shapes.add((96, 32))      # smallest Q8_0 row
    shapes.add((1, 4096))
    return sorted(shapes)


@pytest.mark.parametrize("n,k", _gemv_shapes())
@pytest.mark.parametrize("m", [1, 3, 8, 11])
def test_matmul_q8_matches_oracle(cuda, oracle, n, k, m):
    torch = cuda
    if m > 1 and n * k > 20_000_000:
        pytest.skip("multi-row case covered on the smaller shapes")
    w = synth_q8(7, n * 131 + k, n, k)
    a = synth_f32(8, m * 7 + k, m * k, 1.0)
    want = np.empty(m * n, dtype=np.float32)
    oracle.matmul_q8(ptr(a), ptr(w), ptr(want), m, n, k)
    qs, d = _q8_dev(torch, w, n, k)
    ad = dev(torch, a)
    out = torch.empty(m * n, dtype=torch.float32, device="cuda")
    _capi.check(_lib().jyc_matmul_q8(ad.data_ptr(), qs.data_ptr(), d.data_ptr(), out.data_ptr(),
                                     m, n, k, stream(torch)))
    got = host(out)
    # fp32 re-association only (exact int8*fp16 products): 2e-5 of the row scale
    scale = np.abs(want).max() + 1e-30
    assert np.abs(got - want).max() <= 2e-5 * scale


CHECK_MATMUL_CASES = [
    (1, 1, 1, 1e-4), (2, 2, 2, 1e-4), (4, 4, 4, 1e-4), (8, 8, 8, 1e-4), (16, 16, 16, 1e-4),
    (32, 32, 32, 1e-4), (64, 64, 64, 1e-4), (1, 100, 50, 1e-4), (100, 1, 50, 1e-4),
    (100, 50, 1, 1e-4), (3, 5, 7, 1e-4), (7, 13, 17, 1e-4), (17, 31, 63, 1e-4),
    (33, 65, 129, 1e-4), (128, 128, 128, 1e-3), (256, 256, 256, 1e-3), (512, 512, 512, 1e-3),
    (1, 4096, 1, 1e-4), (4096, 1, 1, 1e-4), (1, 1, 4096, 1e-4),
]


@pytest.mark.parametrize("ci", range(len(CHECK_MATMUL_CASES)))
def test_matmul_f32_check_matmul_cases(cuda, ci):
    """The reference's check_matmul (libs/text/text.h:48-107): same shapes,
    same glibc srand(42+ci)/rand() operands, same double reference and eps."""
    torch = cuda
    m, n, k, eps = CHECK_MATMUL_CASES[ci]
    both = libc_rand_fill(42 + ci, m * k + k * n)
    A, B = both[: m * k], both[m * k:]
    ref = (A.reshape(m, k).astype(np.float64) @ B.reshape(k, n).astype(np.float64)).astype(np.float32)
    Ad, Bd = dev(torch, A), dev(torch, B)
    Bt = torch.empty(n * k, dtype=torch.float32, device="cuda")
    C_ = torch.empty(m * n, dtype=torch.float32, device="cuda")
    lib = _lib()
    _capi.check(lib.jyc_f32_transpose(Bd.data_ptr(), Bt.data_ptr(), k, n, stream(torch)))
    _capi.check(lib.jyc_matmul_f32(Ad.data_ptr(), Bt.data_ptr(), C_.data_ptr(), m, n, k, stream(torch)))
    got = host(C_).reshape(m, n)
    assert np.abs(got - ref).max() <= eps


@pytest.mark.parametrize("n", [512, 896, 2048, 4096, 24, 7, 100])
@pytest.mark.parametrize("rows", [1, 5])
def test_rmsnorm_matches_oracle(cuda, oracle, n, rows):
    torch = cuda
    x = synth_f32(9, n, rows * n, 1.0)
    w = synth_f32(10, n, n, 1.0) + np.float32(1.0)
    want = np.empty_like(x)
    for r in range(rows):
        oracle.rmsnorm(ptr(x[r * n:]), ptr(want[r * n:]), ptr(w), n, f32(1e-5))
    xd, wd = dev(torch, x), dev(torch, w)
    y = torch.empty_like(xd)
    _capi.check(_lib().jyc_rmsnorm(xd.data_ptr(), y.data_ptr(), wd.data_ptr(), rows, n, 1e-5, stream(torch)))
    got = host(y)
    # only the sum-of-squares order differs: a few ulp of the scale
    assert np.abs(got - want).max() <= 4e-7 * np.abs(want).max()


@pytest.mark.parametrize("hd,theta", [(64, 1e4), (64, 1e6), (128, 5e5), (4, 1e4), (32, 1e4), (36, 1e4)])
def test_rope_bit_exact(cuda, oracle, hd, theta):
    torch = cuda
    max_seq, seq, heads, start = 96, 5, 6, 40
    cos, sin = rope_table(max_seq, hd, theta)
    q = synth_f32(11, hd, seq * heads * hd, 1.0)
    want = q.copy()
    oracle.rope_pos(ptr(want), seq, start, heads, hd, ptr(cos), ptr(sin))
    qd, cd, sd = dev(torch, q), dev(torch, cos), dev(torch, sin)
    _capi.check(_lib().jyc_rope_pos(qd.data_ptr(), seq, start, heads, hd, cd.data_ptr(), sd.data_ptr(),
                                    stream(torch)))
    assert np.array_equal(host(qd).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("heads,hd,n", [(4, 64, 3), (2, 64, 1), (8, 128, 2), (1, 4, 5), (3, 36, 2)])
def test_kv_pack_bit_exact(cuda, oracle, heads, hd, n):
    torch = cuda
    src = synth_f32(12, heads * hd, n * heads * hd, 1.0)
    src[:hd] = 0.0          # amax == 0 -> scale 0, bytes 0
    src[hd:2 * hd] *= 1e-9  # amax <= 1e-8 -> scale 0
    want_q = np.empty(n * heads * hd, dtype=np.int8)
    want_s = np.empty(n * heads, dtype=np.float32)
    oracle.kv_pack_q8(ptr(src), ptr(want_q), ptr(want_s), heads, hd, n)
    sd = dev(torch, src)
    q = torch.empty(n * heads * hd, dtype=torch.int8, device="cuda")
    s = torch.empty(n * heads, dtype=torch.float32, device="cuda")
    _capi.check(_lib().jyc_kv_pack_q8(sd.data_ptr(), q.data_ptr(), s.data_ptr(), heads, hd, n, stream(torch)))
    assert np.array_equal(host(q), want_q)
    assert np.array_equal(host(s).view(np.uint32), want_s.view(np.uint32))


ATTN_CASES = [
    # H, KV, hd, seq, start_pos, cap
    (8, 4, 64, 1, 0, 16),      # first token
    (8, 4, 64, 1, 150, 512),   # decode step, c0 heads
    (14, 2, 64, 1, 700, 1024), # c1 heads (group 7)
    (14, 2, 64, 13, 0, 64),    # prefill rows, causal, ragged chunk
    (32, 8, 64, 3, 4000, 4100),  # long context, c2 heads
    (32, 8, 128, 2, 300, 512),   # c3 heads
    (2, 1, 4, 3, 2, 8),          # bind-test shape
]


@pytest.mark.parametrize("H,KV,hd,seq,start,cap", ATTN_CASES)
def test_attention_q8_matches_oracle(cuda, oracle, H, KV, hd, seq, start, cap):
    torch = cuda
    Q = synth_f32(13, H * 1000 + start, seq * H * hd, 1.0)
    K = synth_f32(14, H * 1000 + start, seq * KV * hd, 1.0)
    V = synth_f32(15, H * 1000 + start, seq * KV * hd, 1.0)
    # earlier cache contents: quantised rows of seeded data (same on both sides)
    kc = np.zeros(cap * KV * hd, dtype=np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros(cap * KV, dtype=np.float32)
    vs = np.zeros_like(ks)
    if start:
        kprev = synth_f32(16, hd, start * KV * hd, 1.0)
        vprev = synth_f32(17, hd, start * KV * hd, 1.0)
        oracle.kv_pack_q8(ptr(kprev), ptr(kc), ptr(ks), KV, hd, start)
        oracle.kv_pack_q8(ptr(vprev), ptr(vc), ptr(vs), KV, hd, start)
    dk, dv, dks, dvs = (dev(torch, a) for a in (kc, vc, ks, vs))
    want = np.empty(seq * H * hd, dtype=np.float32)
    assert oracle.attention_q8(ptr(Q), ptr(K), ptr(V), ptr(want), seq, start, H, KV, hd,
                               ptr(kc), ptr(ks), ptr(vc), ptr(vs), cap) == 0
    out = torch.empty(seq * H * hd, dtype=torch.float32, device="cuda")
    Qd, Kd, Vd = dev(torch, Q), dev(torch, K), dev(torch, V)
    _capi.check(_lib().jyc_attention_q8(Qd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), out.data_ptr(),
                                        seq, start, H, KV, hd, dk.data_ptr(), dks.data_ptr(),
                                        dv.data_ptr(), dvs.data_ptr(), cap, stream(torch)))
    got = host(out)
    # int8 cache rows written by both sides: bit-identical
    assert np.array_equal(host(dk), kc) and np.array_equal(host(dv), vc)
    assert np.array_equal(host(dks).view(np.uint32), ks.view(np.uint32))
    assert np.array_equal(host(dvs).view(np.uint32), vs.view(np.uint32))
    # int32 scores are exact; softmax/PV differ by expf ulps and summation order
    assert np.abs(got - want).max() <= 1e-5 * (np.abs(want).max() + 1e-30)


def test_attention_q8_errors(cuda):
    torch = cuda
    lib = _lib()
    buf = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    s = stream(torch)
    assert lib.jyc_attention_q8(p, p, p, p, 1, 0, 6, 4, 64, p, p, p, p, 16, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_attention_q8(p, p, p, p, 4, 14, 8, 4, 64, p, p, p, p, 16, s) == _capi.JYC_ERR_KV_OOM
    assert lib.jyc_attention_q8(p, p, p, p, 0, 0, 8, 4, 64, p, p, p, p, 16, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_attention_q8(p, p, p, p, 1, -1, 8, 4, 64, p, p, p, p, 16, s) == _capi.JYC_ERR_ARG
    assert "capacity" in _capi.last_error() or "start_pos" in _capi.last_error()


@pytest.mark.parametrize("n", [8, 1376, 4864 * 2, 13, 9731])
def test_silu_matches_oracle(cuda, oracle, n):
    torch = cuda
    x = synth_f32(18, n, n, 4.0)
    x[:4] = [0.0, -100.0, 100.0, -87.5]
    want = np.empty_like(x)
    oracle.silu(ptr(x), ptr(want), n)
    xd = dev(torch, x)
    y = torch.empty_like(xd)
    _capi.check(_lib().jyc_silu(xd.data_ptr(), y.data_ptr(), n, stream(torch)))
    got = host(y)
    nv = n // 8 * 8
    # vector body: the reference's own exp polynomial, reproduced bit for bit
    assert np.array_equal(got[:nv].view(np.uint32), want[:nv].view(np.uint32))
    # tail: libm expf vs CUDA expf, a couple of ulp
    if n > nv:
        assert np.allclose(got[nv:], want[nv:], rtol=4e-7, atol=0)


def test_argmax_ties_and_specials(cuda):
    torch = cuda
    lib = _lib()
    v = np.full(100003, -5.0, dtype=np.float32)
    v[777] = 3.0
    v[99999] = 3.0      # tie -> lowest index wins (strict > in generate.h:59-60)
    v[5] = np.nan       # never selected
    v[6] = -np.inf
    vd = dev(torch, v)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    _capi.check(lib.jyc_argmax(vd.data_ptr(), len(v), out.data_ptr(), stream(torch)))
    assert int(host(out)[0]) == 777
    v2 = np.full(17, -np.inf, dtype=np.float32)
    v2d = dev(torch, v2)
    _capi.check(lib.jyc_argmax(v2d.data_ptr(), 17, out.data_ptr(), stream(torch)))
    assert int(host(out)[0]) == 0


# (vocabulary, temperature, repetition penalty)
SAMPLE_CASES = [
    (17, 0.8, 1.0),        # fewer logits than sampler threads
    (1000, 0.0, 1.3),      # penalty + greedy
    (32000, 0.8, 1.3),     # configs[0] vocabulary
    (151936, 0.8, 1.3),    # configs[1] vocabulary
    (151936, 1.7, 1.0),    # flatter distribution
    (128256, 0.3, 2.0),    # configs[3] vocabulary, peaked
]


@pytest.mark.parametrize("V,T,pen", SAMPLE_CASES)
def test_sample_matches_oracle(cuda, oracle, V, T, pen):
    """jyc_sample == jyo_sample (generate.h:50-77) over 12 consecutive draws
    sharing one LCG state: same picks, same rng, the penalised logits bit-exact
    and the probabilities written back within 4e-7 relative (CUDA's expf is
    within 2 ulp, the host libm's within 1) above the smallest normal."""
    torch = cuda
    lib = _lib()
    rs = np.random.default_rng(V * 7 + int(T * 10) + int(pen * 10))
    p0 = 6
    gen = rs.integers(0, min(V, 64), 40)                    # repeats on purpose
    ids = np.concatenate([rs.integers(0, V, p0), gen, [-1, V]]).astype(np.int32)  # two ids outside [0, V)
    ids_d = dev(torch, ids)
    rng_h = C.c_uint(12345)
    rng_d = torch.tensor([12345], dtype=torch.int32, device="cuda")
    out_d = torch.zeros(1, dtype=torch.int32, device="cuda")
    for draw in range(12):
        logits = (rs.standard_normal(V) * 4.0).astype(np.float32)
        logits[rs.integers(0, V)] = 0.0                     # a zero logit: multiplied, stays 0
        want = logits.copy()
        n = len(ids) - (draw % 3)                           # growing / shrinking penalty ranges
        pick = oracle.lib.jyo_sample(want.ctypes.data, V, T, pen, ids.ctypes.data, p0, n, C.byref(rng_h))
        ld = dev(torch, logits)
        _capi.check(lib.jyc_sample(ld.data_ptr(), V, T, pen, ids_d.data_ptr(), p0, n, rng_d.data_ptr(),
                                   out_d.data_ptr(), stream(torch)))
        assert int(host(out_d)[0]) == pick, f"draw {draw}"
        assert int(host(rng_d).view(np.uint32)[0]) == rng_h.value
        got = host(ld)
        if T <= 0.0:
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        else:
            # (+ the smallest normal: denormal results carry no relative
            # accuracy; the sum they join is >= 1, the maximum's own term)
            assert np.all(np.abs(got - want) <= 4e-7 * np.abs(want) + np.float32(2.0 ** -126))


def test_sample_argument_errors(cuda):
    torch = cuda
    lib = _lib()
    buf = torch.zeros(64, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    s = stream(torch)
    assert lib.jyc_sample(p, 0, f32(0.8), f32(1.0), None, 0, 0, p, p, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_sample(p, 16, f32(0.8), f32(1.3), None, 0, 4, p, p, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_sample(p, 16, f32(0.8), f32(1.3), p, 5, 4, p, p, s) == _capi.JYC_ERR_ARG
