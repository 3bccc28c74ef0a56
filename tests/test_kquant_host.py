"""K-quant matmul oracle (oracle/jy_oracle.c jyo_matmul_qk: the block dequant
of libs/matmul_libs/matmul_q.h:47-100 and file_libs/q4/q4_fma.txt, the dot
of dot_row_avx2 / the m > 1 loop, matmul_q.h:111-162) against the reference's
own qmat::matmul_q compiled from its sources (oracle/_ref): bit-identical
outputs for Q4_K, Q5_K and Q6_K, one and several activation rows."""
import ctypes as C
import os

import numpy as np
import pytest

from _kquant import NAMES, Q4K, Q5K, Q6K, kquant_blocks
from oracle.bind import REF_SO, Oracle, Reference


@pytest.fixture(scope="module")
def libs():
    if not os.path.exists(REF_SO):
        pytest.skip("reference harness not built (reference tree absent)")
    o, r = Oracle(), Reference()
    o.lib.jyo_matmul_qk.restype = C.c_int
    return o, r


@pytest.mark.parametrize("qt", [Q4K, Q5K, Q6K], ids=lambda q: NAMES[q])
@pytest.mark.parametrize("m,n,k", [(1, 37, 256), (1, 64, 1024), (3, 29, 512), (8, 16, 768)])
def test_oracle_matches_reference_bit_for_bit(libs, qt, m, n, k):
    o, r = libs
    w = kquant_blocks(qt, n, k, seed=n * 7 + k + qt)
    a = np.random.default_rng(k + m).standard_normal(m * k).astype(np.float32)
    got = np.empty(m * n, np.float32)
    want = np.empty(m * n, np.float32)
    assert o.lib.jyo_matmul_qk(a.ctypes.data, w.ctypes.data, got.ctypes.data, m, n, k, qt) == 0
    r.lib.jyref_matmul_qk(a.ctypes.data, w.ctypes.data, want.ctypes.data, m, n, k, qt)
    assert np.isfinite(want).all()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_oracle_rejects_other_types(libs):
    o, _ = libs
    a = np.zeros(256, np.float32)
    out = np.zeros(1, np.float32)
    w = np.zeros(34 * 8, np.uint8)
    assert o.lib.jyo_matmul_qk(a.ctypes.data, w.ctypes.data, out.ctypes.data, 1, 1, 256, 3) == -1
