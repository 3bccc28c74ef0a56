"""K-quant matmul on the device (jyc_matmul_qk: Q4_K, Q5_K and Q6_K blocks
in the reference's layout) against the oracle's restatement of
qmat::matmul_q (bit-identical to the reference, tests/test_kquant_host.py):
within 2e-5 of max|y| (the dequantised weights are the reference's floats;
only the fp32 summation order differs), one launch per 8 rows of A,
bit-identical on a repeat, and argument errors reported."""
import ctypes as C

import numpy as np
import pytest

from _kquant import NAMES, Q4K, Q5K, Q6K, kquant_blocks
from _util import dev, host, stream
from jieyu_b200 import _capi

pytestmark = pytest.mark.gpu

# (n, k): configs[0]-like down/up rows, a long row, a ragged row count
SHAPES = [(37, 256), (512, 1536), (1000, 4096), (2752, 512)]


@pytest.mark.parametrize("qt", [Q4K, Q5K, Q6K], ids=lambda q: NAMES[q])
@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 5, 8, 11])
def test_kquant_matmul_matches_oracle(cuda, oracle, qt, n, k, m):
    torch = cuda
    lib = _capi.load()
    oracle.lib.jyo_matmul_qk.restype = C.c_int
    w = kquant_blocks(qt, n, k, seed=n * 3 + k + qt)
    a = np.random.default_rng(n + m + k).standard_normal(m * k).astype(np.float32)
    want = np.empty(m * n, np.float32)
    assert oracle.lib.jyo_matmul_qk(a.ctypes.data, w.ctypes.data, want.ctypes.data, m, n, k, qt) == 0
    wd, ad = dev(torch, w), dev(torch, a)
    outs = []
    for _ in range(2):
        out = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
        before = lib.jyc_kernel_launches()
        _capi.check(lib.jyc_matmul_qk(ad.data_ptr(), wd.data_ptr(), out.data_ptr(), m, n, k, qt, stream(torch)))
        assert lib.jyc_kernel_launches() - before == (m + 7) // 8
        outs.append(host(out))
    got = outs[0]
    assert np.isfinite(got).all()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    scale = np.abs(want).max() + 1e-30
    assert np.abs(got - want).max() <= 2e-5 * scale


def test_kquant_matmul_rejects_bad_arguments(cuda):
    torch = cuda
    lib = _capi.load()
    a = torch.zeros(512, dtype=torch.float32, device="cuda")
    w = torch.zeros(2 * 210, dtype=torch.uint8, device="cuda")
    y = torch.zeros(2, dtype=torch.float32, device="cuda")
    s = stream(torch)
    assert lib.jyc_matmul_qk(a.data_ptr(), w.data_ptr(), y.data_ptr(), 1, 1, 384, Q6K, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_matmul_qk(a.data_ptr(), w.data_ptr(), y.data_ptr(), 1, 1, 256, 3, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_matmul_qk(a.data_ptr(), 0, y.data_ptr(), 1, 1, 256, Q4K, s) == _capi.JYC_ERR_ARG
    assert lib.jyc_last_error()
