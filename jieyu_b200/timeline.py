"""Phase timeline of the decode kernel (jyc_model_trace_decode): per layer,
the mean and slowest-CTA duration of every phase of one decode step, read
from the SM clock each CTA records at its phase boundaries.

  python -m jieyu_b200.timeline c3:4096 c1:513     (config:context ...)

A context is set up by prefilling a random prompt of that many tokens; the
traced step then decodes position `context`. Durations are SM clock cycles
converted at --mhz (default: the B200's 1965 MHz boost clock).

Phases per layer (the kernel's order): pro_qkv (residual sum, RMSNorm,
digits), qkv (GEMV), bar1 (grid barrier), attn (attention items), wait (the
O projection's wait for its kv heads), pro_o (split merge + digits), o
(GEMV), bar3, pro_gu, gu, bar4, pro_dn, dn, bar5; and inside a CTA's first
attention item (as warp 0 sees it): a_issue (K/V copies issued, tile
scales requested), a_rq (its query head roped and quantised), a_sync (the
item's other warps: the rest of the query heads, the new K/V rows), a_wait
(its first K/V tile), a_tiles (scores, softmax, P.V), a_merge (the warps'
states merged, split partials written), a_arrive (fence + count).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

PHASES = ["pro_qkv", "qkv", "bar1", "attn", "wait", "pro_o", "o", "bar3", "pro_gu", "gu", "bar4", "pro_dn",
          "dn", "bar5"]
ITEM = ["a_issue", "a_rq", "a_sync", "a_wait", "a_tiles", "a_merge", "a_arrive"]
TRACE_LAYER = 23  # trace points per layer (kMegaTraceLayer)


def trace(name: str, ctx: int, reps: int = 3):
    """Per-CTA phase boundaries [ctas][points] of one traced decode step."""
    import torch

    from . import _capi
    from .model import CONFIGS, DeviceModel, HostWeights, prompt_ids, with_max_seq
    cfg = CONFIGS[name]
    cfg = with_max_seq(cfg, max(cfg.max_seq, ctx + 64))
    hw = HostWeights.synthetic(cfg)
    m = DeviceModel(hw)
    lib = _capi.load()
    st = torch.cuda.Stream()
    s = st.cuda_stream
    ids = torch.from_numpy(prompt_ids(cfg, n=ctx)).cuda()
    m.prefill_device(ids.data_ptr(), ctx, s)
    m.decode_device(4, s)
    st.synchronize()
    npts = lib.jyc_model_trace_points(m.h)
    out = np.zeros(1024 * npts, np.int64)
    for _ in range(reps):  # the last of a few repeats (warm caches, clocks)
        n = _capi.check(lib.jyc_model_trace_decode(m.h, s, out.ctypes.data, out.size))
    tr = out[: n * npts].reshape(n, npts).astype(np.float64)
    m.close()
    return cfg, tr


def summarize(cfg, tr, mhz: float) -> str:
    us = 1.0 / mhz
    L = cfg.layers
    npts = tr.shape[1]
    th = 1 + L * TRACE_LAYER
    step = (tr[:, th + 2] - tr[:, 0]) * us
    rows = {}
    for l in range(L):
        tb = 1 + l * TRACE_LAYER
        prev = tr[:, 0] if l == 0 else tr[:, tb - TRACE_LAYER + 13]
        pts = [prev] + [tr[:, tb + i] for i in range(14)]
        for i, nm in enumerate(PHASES):
            d = (pts[i + 1] - pts[i]) * us
            rows.setdefault(nm, []).append((d.mean(), d.max()))
        a = tr[:, tb + 14: tb + 14 + len(ITEM) + 1]
        ok = a[:, 0] > 0
        if ok.any():
            for i, nm in enumerate(ITEM):
                d = (a[ok, i + 1] - a[ok, i]) * us
                rows.setdefault(nm, []).append((d.mean(), d.max()))
    lines = [f"{cfg.name}: one decode step {np.median(step):.1f} us (median CTA), {step.max():.1f} us (slowest)"]
    per_layer = sum(np.mean([r[0] for r in rows[nm]]) for nm in PHASES)
    lines.append(f"per layer, mean over layers: {per_layer:.2f} us")
    lines.append("| phase | mean over CTAs (us) | slowest CTA (us) |")
    lines.append("|---|---|---|")
    for nm in PHASES + ITEM:
        if nm in rows:
            v = np.array(rows[nm])
            lines.append(f"| {nm} | {v[:, 0].mean():.2f} | {v[:, 1].mean():.2f} |")
    hp = (tr[:, th] - tr[:, th - TRACE_LAYER + 13]) * us
    hc = (tr[:, th + 1] - tr[:, th]) * us
    hb = (tr[:, th + 2] - tr[:, th + 1]) * us
    lines.append(f"| head: prologue / GEMV + argmax / barrier | {hp.mean():.2f} / {hc.mean():.2f} / {hb.mean():.2f} "
                 f"| {hp.max():.2f} / {hc.max():.2f} / {hb.max():.2f} |")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("cases", nargs="+", help="config:context, e.g. c3:4096")
    ap.add_argument("--mhz", type=float, default=1965.0)
    args = ap.parse_args(argv)
    for spec in args.cases:
        name, ctx = spec.split(":")
        cfg, tr = trace(name, int(ctx))
        print(summarize(cfg, tr, args.mhz))
        print()
    return 0


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.exit(main())
