"""Tensor-core (tcgen05) matmul parity: jyc_matmul_q8 with 16 or more rows of
A runs on the tcgen05 tiles (exact fp16 hi/lo splits of the dequantised
weights and of the activations, fp32 accumulation in tensor memory). It must
match the oracle's qmat::matmul_q restatement (libs/matmul_libs/matmul_q.h:
101-143, bit-identical to the reference) within the same 2e-5 of max|y| as the
GEMV path: both are exact products summed in fp32 in another order.
"""
import numpy as np
import pytest

from _util import dev, host, ptr, stream
from jieyu_b200 import _capi
from jieyu_b200.model import synth_f32, synth_q8

pytestmark = pytest.mark.gpu

# (n, k): configs[0] QKV / gate-up (n % 128 != 0) / down (k % 64 == 32),
# configs[1] QKV (split K) and down (long K), a small vocabulary head.
SHAPES = [(1024, 512), (2752, 512), (512, 1376), (1152, 896), (896, 4864), (32000, 512), (128, 32)]


def _q8_dev(torch, blocks, n, k):
    lib = _capi.load()
    b = dev(torch, blocks)
    qs = torch.empty(n * k, dtype=torch.uint8, device="cuda")
    d = torch.empty(n * (k // 32), dtype=torch.int16, device="cuda")
    _capi.check(lib.jyc_q8_repack(b.data_ptr(), n, k, qs.data_ptr(), d.data_ptr(), stream(torch)))
    return qs, d


def _run(torch, oracle, n, k, m, a):
    w = synth_q8(17, n * 7 + k, n, k)
    want = np.empty(m * n, dtype=np.float32)
    oracle.matmul_q8(ptr(a), ptr(w), ptr(want), m, n, k)
    qs, d = _q8_dev(torch, w, n, k)
    ad = dev(torch, a)
    out = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
    launches = _capi.load().jyc_kernel_launches()
    _capi.check(_capi.load().jyc_matmul_q8(ad.data_ptr(), qs.data_ptr(), d.data_ptr(), out.data_ptr(),
                                           m, n, k, stream(torch)))
    assert _capi.load().jyc_kernel_launches() - launches == 3  # row exponents + split + tcgen05 GEMM
    got = host(out)
    assert _capi.load().jyc_device_error(1) == 0
    return got, want


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", [16, 37, 64, 128, 200])
def test_tc_matmul_matches_oracle(cuda, oracle, n, k, m):
    torch = cuda
    if m > 64 and n * k > 5_000_000:
        pytest.skip("large-row cases covered on the smaller shapes")
    a = synth_f32(18, m * 5 + k, m * k, 1.0)
    got, want = _run(torch, oracle, n, k, m, a)
    assert np.isfinite(got).all()
    scale = np.abs(want).max() + 1e-30
    err = np.abs(got - want).max()
    assert err <= 2e-5 * scale, f"max|d| {err} vs {scale}"


def test_tc_matmul_wide_dynamic_range(cuda, oracle):
    """Rows of very different magnitude, zero rows of A and an activation
    column far below the row maximum: the per-row / per-token power-of-two
    scales keep every product exact."""
    torch = cuda
    n, k, m = 256, 512, 32
    a = synth_f32(19, 3, m * k, 1.0).reshape(m, k)
    a[3] = 0.0
    a[5] *= 1e-6
    a[7, ::2] *= 1e-4
    a = np.ascontiguousarray(a.reshape(-1))
    got, want = _run(torch, oracle, n, k, m, a)
    got = got.reshape(m, n)
    want = want.reshape(m, n)
    assert np.all(got[3] == 0.0)
    for r in range(m):
        scale = np.abs(want[r]).max() + 1e-30
        assert np.abs(got[r] - want[r]).max() <= 2e-5 * scale, r
