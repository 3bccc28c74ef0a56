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
