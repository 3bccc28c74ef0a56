"""Few-row Q8_0 matmul (2..15 rows of A through jyc_matmul_q8): activations in
registers, one 512-column K slice per warp unit, slices summed in order by
the last unit of a row range. It must match the oracle's qmat::matmul_q
restatement (libs/matmul_libs/matmul_q.h:101-143, bit-identical to the
reference) within 2e-5 of max|y| (exact int8 x fp16 products, fp32 sums in
another order), launch one kernel per 8 rows, and give bit-identical results
run after run (the split-K sum has a fixed order).
"""
import numpy as np
import pytest

from _util import dev, host, ptr, stream
from jieyu_b200 import _capi
from jieyu_b200.model import synth_f32, synth_q8

pytestmark = pytest.mark.gpu

# (n, k): one partial slice (k < 512), ragged last slice (1376 = 2 x 512 + 352),
# 16 slices (8192), 28 slices (configs[3] down), odd row counts, tiny n.
SHAPES = [(96, 32), (1000, 1376), (333, 8192), (64, 14336), (2, 512), (4099, 2048)]


def _q8_dev(torch, blocks, n, k):
    lib = _capi.load()
    b = dev(torch, blocks)
    qs = torch.empty(n * k, dtype=torch.uint8, device="cuda")
    d = torch.empty(n * (k // 32), dtype=torch.int16, device="cuda")
    _capi.check(lib.jyc_q8_repack(b.data_ptr(), n, k, qs.data_ptr(), d.data_ptr(), stream(torch)))
    return qs, d


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [2, 4, 5, 8, 9, 15])
def test_skinny_matmul_matches_oracle(cuda, oracle, n, k, m):
    torch = cuda
    lib = _capi.load()
    w = synth_q8(23, n * 11 + k, n, k)
    a = synth_f32(24, m * 3 + k, m * k, 1.0)
    want = np.empty(m * n, dtype=np.float32)
    oracle.matmul_q8(ptr(a), ptr(w), ptr(want), m, n, k)
    qs, d = _q8_dev(torch, w, n, k)
    ad = dev(torch, a)
    outs = []
    for _ in range(2):
        out = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
        before = lib.jyc_kernel_launches()
        _capi.check(lib.jyc_matmul_q8(ad.data_ptr(), qs.data_ptr(), d.data_ptr(), out.data_ptr(),
                                      m, n, k, stream(torch)))
        assert lib.jyc_kernel_launches() - before == (m + 7) // 8
        outs.append(host(out))
    got = outs[0]
    assert np.isfinite(got).all()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "not deterministic"
    scale = np.abs(want).max() + 1e-30
    err = np.abs(got - want).max()
    assert err <= 2e-5 * scale, f"max|d| {err} vs {scale}"
