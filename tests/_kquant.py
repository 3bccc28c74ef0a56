"""Seeded K-quant weight blocks for the tests (random quant bytes; the fp16
scale fields set to finite values so every block dequantises to finite
weights)."""
import numpy as np

Q4K, Q5K, Q6K = 0, 1, 2
BLOCK_BYTES = {Q4K: 144, Q5K: 176, Q6K: 210}
NAMES = {Q4K: "q4_K", Q5K: "q5_K", Q6K: "q6_K"}


def kquant_blocks(qt: int, n: int, k: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    nb = n * (k // 256)
    bb = BLOCK_BYTES[qt]
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    d = rng.uniform(2.0 ** -12, 2.0 ** -7, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if qt == Q6K:
        b[:, 208:210] = d
    else:
        dmin = rng.uniform(2.0 ** -12, 2.0 ** -8, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        b[:, 0:2] = d
        b[:, 2:4] = dmin
    return np.ascontiguousarray(b.reshape(-1))
