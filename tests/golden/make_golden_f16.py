"""Generates tests/golden/f16.json by running the REFERENCE itself
(oracle/_ref/libjyref.so, the jieyu headers compiled unmodified, JIEYU_ISA=fma)
on seeded fp16 weights: the matmul_f16 digests of a few shapes (through the
reference's own matmul_w dispatch, wmat_kernel.h:9-16 -> matmul_f16.h:19-41)
and the greedy sequence of the configs[0] shape with every linear matrix, the
LM head and the embedding in fp16 (HostWeights.synthetic_f16). Run from the
repository root, where the reference tree exists:

    make -C oracle all REF=<reference tree> && python tests/golden/make_golden_f16.py
"""
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.bind import Reference  # noqa: E402
from jieyu_b200.model import CONFIGS, HostWeights, prompt_ids, synth_f32  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
# (m, n, k): n % 8 != 0 exercises the reference's scalar tail columns
F16_CASES = [(1, 64, 512), (3, 40, 96), (5, 7, 32), (2, 13, 5), (1, 1376, 512), (9, 100, 72), (1, 4096, 2048)]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def f16_inputs(m, n, k):
    """Seeded activations (std 1) and fp16 weights [k][n] (std 0.05, rounded to nearest even)."""
    a = synth_f32(120, m * 31 + n, m * k, 1.0)
    b = synth_f32(121, n * 31 + k, k * n, 0.05).astype(np.float16).view(np.uint16)
    return a, b


def main():
    ref = Reference("fma", 0)
    g = {"isa": "fma", "ops": {}}
    for m, n, k in F16_CASES:
        a, b = f16_inputs(m, n, k)
        c = np.empty(m * n, np.float32)
        ref.matmul_f16(a.ctypes.data, b.ctypes.data, c.ctypes.data, m, n, k)
        g["ops"][f"f16_{m}_{n}_{k}"] = sha(c)
    c0 = CONFIGS["c0"]
    hw = HostWeights.synthetic_f16(c0)
    pr = prompt_ids(c0)
    ids = ref.generate(hw.desc, pr, 64, max_seq=c0.max_seq)
    g["c0_f16"] = {"seed": 1234, "prompt": [int(x) for x in pr], "greedy": [int(x) for x in ids]}
    with open(os.path.join(OUT, "f16.json"), "w") as f:
        json.dump(g, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
