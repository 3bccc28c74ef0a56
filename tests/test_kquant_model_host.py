"""A model in the reference's K-quant formats (Q4_K / Q5_K / Q6_K weights
mixed per matrix, Q6_K head and embedding) through the oracle's generate
(matmul_w / wmat_row with the K-quant restatement) gives the same greedy ids
as the reference's own generate() (libs/model_libs/generate.h:90-112,
compiled from its sources)."""
import os

import numpy as np
import pytest

from _kquant import kquant_model
from oracle.bind import REF_SO, Oracle, Reference


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference harness not built")
def test_kquant_model_oracle_matches_reference():
    hw = kquant_model()
    prompt = np.array([3, 17, 255, 42, 7, 99, 150, 8], np.int32)
    want = Reference().generate(hw.desc, prompt, 12, max_seq=hw.cfg.max_seq)
    got = Oracle().generate(hw.desc, prompt, 12, max_seq=hw.cfg.max_seq)
    assert len(want) == len(prompt) + 12
    assert list(got) == list(want)
    assert len(set(int(x) for x in want[len(prompt):])) > 1  # not a degenerate model


def test_kquant_in_place_byte_accounting():
    """All layer matrices K-quant: the bytes a decode token streams are the
    blocks' own (read in place), not 4 bytes per weight; the LM head and
    embedding row stay fp32 (dequantised once at upload)."""
    hw = kquant_model()
    cfg = hw.cfg
    D, F, qd, kvd = cfg.hidden, cfg.inter, cfg.q_dim, cfg.kv_dim
    names = ("q", "k", "v", "o", "gate", "up", "down")
    blocks = sum(hw.t[f"{n}.{l}"].nbytes for l in range(cfg.layers) for n in names)
    bb = {0: 144, 1: 176, 2: 210}
    dims = {"q": (qd, D), "k": (kvd, D), "v": (kvd, D), "o": (D, qd), "gate": (F, D), "up": (F, D), "down": (D, F)}
    assert blocks == sum(n * (k // 256) * bb[hw.qt[f"{m}.{l}"]] for l in range(cfg.layers) for m, (n, k) in dims.items())
    want = blocks + cfg.layers * 2 * D * 4 + cfg.vocab * D * 4 + 4 * D + D * 4
    assert abs(hw.weight_bytes_per_token() - want) <= 1e-9 * want
