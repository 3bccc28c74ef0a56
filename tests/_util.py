"""Shared helpers of the test suite (device buffers via torch, tolerances)."""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Logit tolerance of the north-star parity bar: max|dlogit| <= 1e-3 * max|logit|.
LOGIT_TOL = 1e-3


def golden(name: str) -> dict:
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def f32(x) -> C.c_float:
    return C.c_float(x)


def dev(torch, a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream(torch) -> int:
    return torch.cuda.current_stream().cuda_stream


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def libc_rand_fill(seed: int, n: int) -> np.ndarray:
    """(rand() % 2000 - 1000) / 1000.0f with glibc srand/rand, as check_matmul
    (libs/text/text.h:82-84) fills its operands."""
    libc = C.CDLL("libc.so.6")
    libc.srand(seed)
    r = np.fromiter((libc.rand() for _ in range(n)), dtype=np.int64, count=n)
    return ((r % 2000 - 1000).astype(np.float32) / np.float32(1000.0)).astype(np.float32)
