"""Generates tests/golden/longctx.json from the reference itself (oracle/_ref,
the jieyu headers compiled unmodified): teacher-forced decode steps at long
KV contexts, for configs[2] (Q8_0 and fp32 weights) at contexts 4096 and
16384 and for configs[3] at 4096.

The reference's prefill of such a prompt would take hours on the scalar m>1
path, so the context is a seeded int8 K/V cache (oracle.synth.context_kv)
written into the reference's own __KVcache; then generate_cached's step body
(forward_cached over one token + the LM head, generate.h:40-49) runs at
positions ctx, ctx+1, ... fed with the fma path's own argmax. Per step the
fixture keeps the argmax, the top-2 gap, max|logit|, a digest of the logits,
and the reference's own scalar-vs-fma spread (max|dlogit| / max|logit| on
identical inputs), which the device tests use for their tolerance.

  python tests/golden/make_golden_longctx.py      (needs oracle/_ref built)
"""
import ctypes as C
import hashlib
import json
import os
import sys
from dataclasses import replace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from jieyu_b200.model import CONFIGS, HostWeights, prompt_ids  # noqa: E402
from oracle.bind import Reference  # noqa: E402
from oracle.synth import context_kv  # noqa: E402

STEPS = 3
# (config, context, layers): the whole model (where the reference's own
# scalar-vs-fma spread is large: chaotic growth of fp32 rounding differences
# over the layers through the int8 KV quantisation) and its first two layers
# (same weights, full width and vocabulary: a spread far below 1e-3, so the
# device can be held to the north-star bar there)
CASES = [("c2", 4096, 0), ("c2", 16384, 0), ("c2f", 4096, 0), ("c2f", 16384, 0), ("c3", 4096, 0),
         ("c2", 4096, 2), ("c2", 16384, 2), ("c2f", 16384, 2), ("c3", 4096, 2), ("c3", 16384, 2)]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def long_cfg(key, ctx, layers=0):
    """The config with a context of `ctx` positions plus the steps (and only
    its first `layers` layers when layers > 0)."""
    cfg = replace(CONFIGS[key], max_seq=ctx + 16)
    return replace(cfg, layers=layers, name=f"{cfg.name}_{layers}l") if layers else cfg


def case_name(key, ctx, layers=0):
    return f"{key}_{ctx}" + (f"_{layers}l" if layers else "")


def first_token(cfg):
    return int(prompt_ids(cfg, n=1, index=7)[0])


def run(chk, hw, ctx, toks):
    """STEPS + 1 single-token steps from a cache holding the seeded context;
    feeds `toks` when given, else the step's own argmax."""
    cfg = hw.cfg
    cache = chk.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    for l, k, ks, v, vs in context_kv(cfg.layers, ctx, cfg.kv_heads, cfg.head_dim):
        chk.cache_write(cache, l, ctx, k.ctypes.data, ks.ctypes.data, v.ctypes.data, vs.ctypes.data)
    logits = np.empty(cfg.vocab, np.float32)
    out, fed = [], []
    tok = first_token(cfg)
    for s in range(STEPS + 1):
        fed.append(tok)
        t = np.array([tok], np.int32)
        assert chk.forward_logits(C.byref(hw.desc), cache, t.ctypes.data, 1, ctx + s, logits.ctypes.data, None) == 0
        out.append(logits.copy())
        tok = toks[s] if toks is not None else int(np.argmax(logits))
    chk.cache_free(cache)
    return out, fed


def main():
    res = {}
    for key, ctx, layers in CASES:
        hw = HostWeights.synthetic(long_cfg(key, ctx, layers))
        fma, fed = run(Reference("fma", 0), hw, ctx, None)
        toks = [int(np.argmax(x)) for x in fma]
        scalar, _ = run(Reference("scalar", 0), hw, ctx, toks)
        Reference("fma", 0)  # the library's ISA switch is global: leave it on fma
        rows = []
        for a, b in zip(fma, scalar):
            top = np.argsort(-a.astype(np.float64), kind="stable")[:5]
            rows.append({"argmax": int(np.argmax(a)), "gap": float(a[top[0]] - a[top[1]]),
                         "amax": float(np.abs(a).max()), "sha": sha(a), "top5": [int(i) for i in top],
                         "isa_spread": float(np.abs(a - b).max() / np.abs(a).max())})
        res[case_name(key, ctx, layers)] = {"config": key, "ctx": ctx, "layers": hw.cfg.layers,
                                            "max_seq": hw.cfg.max_seq, "fed": fed, "steps": rows}
        print(key, ctx, layers, [r["argmax"] for r in rows], [round(r["isa_spread"], 5) for r in rows], flush=True)
        del hw
    with open(os.path.join(HERE, "longctx.json"), "w") as f:
        json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
