"""jyc_attention_q8_noalloc (fixed scratch, no allocation) against
jyc_attention_q8 (stream-ordered scratch): same outputs and cache bytes on two
consecutive calls, within the attention op tests' tolerance. Collected last
(file name) so it also runs after every other GPU test in one process."""
import numpy as np
import pytest

from _util import dev, host, stream
from jieyu_b200 import _capi
from jieyu_b200.model import synth_f32

pytestmark = pytest.mark.gpu

# (H, KV, head_dim, start, first seq, second seq, cache capacity)
CASES = [
    (14, 2, 64, 100, 5, 1, 1024),   # configs[1] heads, decode-sized second call
    (8, 4, 64, 0, 9, 3, 512),       # configs[0] heads, prompt then a short step
    (32, 8, 128, 700, 1, 1, 4352),  # configs[3] heads
    (32, 8, 64, 40, 20, 20, 512),   # 20 rows: the 8-row loop reuses the scratch inside one call
]


def _run(lib, torch, fn, H, KV, hd, start, seqs, cap):
    """Two consecutive calls of `fn` on one cache; returns outputs and cache."""
    kc = torch.zeros(cap * KV * hd, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(cap * KV, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    outs = []
    pos = start
    for i, seq in enumerate(seqs):
        Q = dev(torch, synth_f32(40 + i, H * 1000 + pos, seq * H * hd, 1.0))
        K = dev(torch, synth_f32(50 + i, H * 1000 + pos, seq * KV * hd, 1.0))
        V = dev(torch, synth_f32(60 + i, H * 1000 + pos, seq * KV * hd, 1.0))
        out = torch.empty(seq * H * hd, dtype=torch.float32, device="cuda")
        _capi.check(fn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), seq, pos, H, KV, hd,
                       kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(), cap, stream(torch)))
        outs.append(host(out))
        pos += seq
    return outs, [host(t) for t in (kc, vc, ks, vs)]


@pytest.mark.parametrize("H,KV,hd,start,s1,s2,cap", CASES)
def test_noalloc_attention_matches_allocating_entry(cuda, H, KV, hd, start, s1, s2, cap):
    torch = cuda
    lib = _capi.load()
    want, wcache = _run(lib, torch, lib.jyc_attention_q8, H, KV, hd, start, (s1, s2), cap)
    got, gcache = _run(lib, torch, lib.jyc_attention_q8_noalloc, H, KV, hd, start, (s1, s2), cap)
    # the same kernels with the same split plan: bit-identical outputs
    for g, w in zip(got, want):
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
    for g, w in zip(gcache, wcache):
        assert np.array_equal(g.view(np.uint8), w.view(np.uint8))


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    torch = cuda
    lib = _capi.load()
    buf = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    s = stream(torch)
    # 40 heads x 256 dims = 10240 > 8192 query elements per row
    assert lib.jyc_attention_q8_noalloc(p, p, p, p, 1, 0, 40, 40, 256, p, p, p, p, 16, s) == _capi.JYC_ERR_ARG
    assert "fixed scratch" in _capi.last_error()
    # split partials: 8 rows x 128 heads x 64 dims x 17 splits (start 1024,
    # 4 kv heads) = 1,114,112 floats > 1,048,576
    assert lib.jyc_attention_q8_noalloc(p, p, p, p, 1, 1024, 128, 4, 64, p, p, p, p, 1025, s) == _capi.JYC_ERR_ARG
    assert "fixed scratch" in _capi.last_error()
    # arrival counters: one per kv head, 256 of them
    assert lib.jyc_attention_q8_noalloc(p, p, p, p, 1, 0, 257, 257, 4, p, p, p, p, 16, s) == _capi.JYC_ERR_ARG
    assert "fixed scratch" in _capi.last_error()
    # the usual argument checks still apply
    assert lib.jyc_attention_q8_noalloc(p, p, p, p, 4, 14, 8, 4, 64, p, p, p, p, 16, s) == _capi.JYC_ERR_KV_OOM
