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


def kquant_blocks_scaled(qt: int, n: int, k: int, seed: int, lo: float, hi: float) -> np.ndarray:
    """Like kquant_blocks, with d (and dmin) drawn from [lo, hi]."""
    rng = np.random.default_rng(seed)
    nb = n * (k // 256)
    bb = BLOCK_BYTES[qt]
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    d = rng.uniform(lo, hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if qt == Q6K:
        b[:, 208:210] = d
    else:
        b[:, 0:2] = d
        b[:, 2:4] = rng.uniform(lo, hi, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return np.ascontiguousarray(b.reshape(-1))


def kquant_model():
    """A small model in the K-quant formats of the reference's downloads,
    mixed per matrix as Q4_K_M files mix them: Q4_K / Q5_K / Q6_K layer
    weights, a Q6_K LM head and embedding (zero-centred, so tokens differ);
    unit norms."""
    from jieyu_b200.model import Config, HostWeights, rope_table
    cfg = Config("kq_tiny", 256, 2, 4, 2, 64, 512, 300, 1e4, "kq", "q8", False, 128, 16, 16)
    D, F, V, qd, kvd = cfg.hidden, cfg.inter, cfg.vocab, cfg.q_dim, cfg.kv_dim
    kinds = {"q": Q4K, "k": Q5K, "v": Q6K, "o": Q4K, "gate": Q4K, "up": Q5K, "down": Q6K}
    dims = {"q": (qd, D), "k": (kvd, D), "v": (kvd, D), "o": (D, qd), "gate": (F, D), "up": (F, D), "down": (D, F)}
    t, qt = {}, {}
    ones = np.ones(D, np.float32)
    for l in range(cfg.layers):
        t[f"rms1.{l}"] = ones
        t[f"rms2.{l}"] = ones
        for i, (key, q) in enumerate(kinds.items()):
            n, k = dims[key]
            lo, hi = (2.0 ** -17, 2.0 ** -15) if q == Q6K else (2.0 ** -13, 2.0 ** -11)
            t[f"{key}.{l}"] = kquant_blocks_scaled(q, n, k, 100 * l + i, lo, hi)
            qt[f"{key}.{l}"] = q
    t["head"] = kquant_blocks_scaled(Q6K, V, D, 900, 2.0 ** -15, 2.0 ** -13)
    qt["head"] = Q6K
    t["embed"] = kquant_blocks_scaled(Q6K, V, D, 901, 2.0 ** -12, 2.0 ** -10)
    qt["embed"] = Q6K
    t["final_norm"] = ones
    cos, sin = rope_table(cfg.max_seq, cfg.head_dim, cfg.theta)
    return HostWeights(cfg, t, cos, sin, qtypes=qt)
