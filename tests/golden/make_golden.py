"""Generates the golden fixtures in this directory by running the REFERENCE
itself (oracle/_ref/libjyref.so, the jieyu headers compiled unmodified) on
seeded inputs. Run from the repository root, where the reference tree exists:

    make -C oracle all REF=<reference tree> && python tests/golden/make_golden.py

The fixtures hold seeds, token ids, a few values and SHA-256 digests of
outputs, never large tensors. JIEYU_ISA=fma pins the reference's code path
(AVX2+FMA; its int8 dot is exact either way).
"""
import ctypes as C
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.bind import Reference  # noqa: E402
from jieyu_b200.model import (CONFIGS, HostWeights, prompt_ids, rope_table,  # noqa: E402
                              synth_f32, synth_ids, synth_q8)

OUT = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def p(a):
    return a.ctypes.data


# Operator cases: inputs are seeded (jyc_synth_*), outputs are the reference's.
Q8_CASES = [(1, 64, 512), (3, 40, 96), (1, 1376, 512), (5, 7, 32), (1, 896, 4864), (2, 128, 896)]
F32_CASES = [(1, 1, 1), (7, 13, 5), (1, 4096, 1), (33, 17, 9), (4, 64, 64), (1, 96, 2048)]
RMS_CASES = [512, 896, 2048, 4096, 7, 24, 100]
SILU_CASES = [8, 1376, 13, 9731]
ROPE_CASES = [(64, 64, 1e4), (16, 128, 5e5), (8, 4, 1e4), (40, 36, 1e6)]
ATTN_CASES = [(8, 4, 64, 1, 0, 16), (8, 4, 64, 1, 150, 512), (14, 2, 64, 13, 0, 64),
              (32, 8, 128, 2, 300, 512), (2, 1, 4, 3, 2, 8)]


def op_inputs_q8(m, n, k):
    return synth_q8(101, n * 131 + k, n, k), synth_f32(102, m * 7 + k, m * k, 1.0)


def op_inputs_f32(m, n, k):
    return synth_f32(103, m * 31 + n, m * k, 1.0), synth_f32(104, n * 31 + k, k * n, 1.0)


def attn_inputs(H, KV, hd, seq, start, cap, ref):
    Q = synth_f32(105, H * 1000 + start, seq * H * hd, 1.0)
    K = synth_f32(106, H * 1000 + start, seq * KV * hd, 1.0)
    V = synth_f32(107, H * 1000 + start, seq * KV * hd, 1.0)
    kc = np.zeros(cap * KV * hd, np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros(cap * KV, np.float32)
    vs = np.zeros_like(ks)
    if start:
        kp = synth_f32(108, hd, start * KV * hd, 1.0)
        vp = synth_f32(109, hd, start * KV * hd, 1.0)
        ref.kv_pack_q8(p(kp), p(kc), p(ks), KV, hd, start)
        ref.kv_pack_q8(p(vp), p(vc), p(vs), KV, hd, start)
    return Q, K, V, kc, ks, vc, vs


def run_ops(chk):
    """Runs every operator case on `chk` (Reference or Oracle); returns digests."""
    res = {}
    for m, n, k in Q8_CASES:
        w, a = op_inputs_q8(m, n, k)
        c = np.empty(m * n, np.float32)
        chk.matmul_q8(p(a), p(w), p(c), m, n, k)
        res[f"q8_{m}_{n}_{k}"] = sha(c)
    for m, n, k in F32_CASES:
        A, B = op_inputs_f32(m, n, k)
        c = np.empty(m * n, np.float32)
        chk.matmul_f32(m, n, k, p(A), p(B), p(c))
        res[f"f32_{m}_{n}_{k}"] = sha(c)
    for n in RMS_CASES:
        x = synth_f32(110, n, n, 1.0)
        w = synth_f32(111, n, n, 1.0)
        y = np.empty(n, np.float32)
        chk.rmsnorm(p(x), p(y), p(w), n, C.c_float(1e-5))
        res[f"rms_{n}"] = sha(y)
    for n in SILU_CASES:
        x = synth_f32(112, n, n, 4.0)
        y = np.empty(n, np.float32)
        chk.silu(p(x), p(y), n)
        res[f"silu_{n}"] = sha(y)
    for ms, hd, th in ROPE_CASES:
        cs = np.empty(ms * hd // 2, np.float32)
        sn = cs.copy()
        chk.rope_table(ms, hd, C.c_float(th), p(cs), p(sn))
        q = synth_f32(113, hd, 3 * 5 * hd, 1.0)
        chk.rope_pos(p(q), 3, ms - 4, 5, hd, p(cs), p(sn))
        res[f"ropetab_{ms}_{hd}_{th:g}"] = sha(np.concatenate([cs, sn]))
        res[f"rope_{ms}_{hd}_{th:g}"] = sha(q)
    for H, KV, hd, seq, start, cap in ATTN_CASES:
        Q, K, V, kc, ks, vc, vs = attn_inputs(H, KV, hd, seq, start, cap, chk)
        out = np.empty(seq * H * hd, np.float32)
        rc = chk.attention_q8(p(Q), p(K), p(V), p(out), seq, start, H, KV, hd, p(kc), p(ks),
                              p(vc), p(vs), cap)
        assert rc == 0
        res[f"attn_{H}_{KV}_{hd}_{seq}_{start}"] = sha(out)
        res[f"attnkv_{H}_{KV}_{hd}_{seq}_{start}"] = sha(np.concatenate(
            [kc.view(np.uint8), vc.view(np.uint8), ks.view(np.uint8), vs.view(np.uint8)]))
    return res


def teacher_forced(chk, hw, prompt, steps):
    """Prefill + `steps` single-token steps fed with the reference's own argmax;
    per step: argmax id, top-2 gap, max|logit| and a digest of the logits."""
    cfg = hw.cfg
    cache = chk.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
    logits = np.empty(cfg.vocab, np.float32)
    ids = np.ascontiguousarray(prompt, np.int32)
    rows = []
    pos = 0
    tok = ids
    for s in range(steps + 1):
        rc = chk.forward_logits(C.byref(hw.desc), cache, p(tok), len(tok), pos, p(logits), None)
        assert rc == 0
        pos += len(tok)
        top = np.argsort(-logits.astype(np.float64), kind="stable")[:2]
        rows.append({"argmax": int(np.argmax(logits)), "gap": float(logits[top[0]] - logits[top[1]]),
                     "amax": float(np.abs(logits).max()), "sha": sha(logits),
                     "top5": [int(i) for i in np.argsort(-logits, kind="stable")[:5]]})
        tok = np.array([rows[-1]["argmax"]], np.int32)
    kv = {}
    n = pos
    k = np.empty(n * cfg.kv_dim, np.int8)
    v = np.empty_like(k)
    ks = np.empty(n * cfg.kv_heads, np.float32)
    vs = np.empty_like(ks)
    for layer in (0, cfg.layers - 1):
        chk.cache_read(cache, layer, n, p(k), p(ks), p(v), p(vs))
        kv[str(layer)] = sha(np.concatenate([k.view(np.uint8), v.view(np.uint8),
                                             ks.view(np.uint8), vs.view(np.uint8)]))
    chk.cache_free(cache)
    return rows, kv


def isa_spread(hw, prompt, steps):
    """The reference's own scalar path against its fma path on identical
    inputs (both fed the fma path's argmax): per step max|dlogit| / max|logit|,
    and per layer (0, last) the fraction of int8 K/V bytes that differ. The
    device parity tests allow max(1e-3, 1.5 x) this spread."""
    cfg = hw.cfg
    outs, kvs = [], []
    toks = None
    for isa in ("fma", "scalar"):
        chk = Reference(isa, 0)
        cache = chk.cache_create(cfg.layers, cfg.max_seq, cfg.kv_heads, cfg.head_dim)
        logits = np.empty(cfg.vocab, np.float32)
        seq = [np.ascontiguousarray(prompt, np.int32)]
        if toks is not None:
            seq += [np.array([t], np.int32) for t in toks]
        got, tk = [], []
        pos = 0
        for s in range(steps + 1):
            tok = seq[s] if s < len(seq) else np.array([tk[-1]], np.int32)
            assert chk.forward_logits(C.byref(hw.desc), cache, p(tok), len(tok), pos, p(logits), None) == 0
            pos += len(tok)
            got.append(logits.copy())
            tk.append(int(np.argmax(logits)))
        if toks is None:
            toks = tk[:steps]
        n = pos
        lay = {}
        for layer in (0, cfg.layers - 1):
            k = np.empty(n * cfg.kv_dim, np.int8)
            v = np.empty_like(k)
            ks = np.empty(n * cfg.kv_heads, np.float32)
            vs = np.empty_like(ks)
            chk.cache_read(cache, layer, n, p(k), p(ks), p(v), p(vs))
            lay[layer] = (k.copy(), v.copy())
        chk.cache_free(cache)
        outs.append(got)
        kvs.append(lay)
    Reference("fma", 0)  # the library's ISA switch is global: leave it on fma
    logit = [float(np.abs(a - b).max() / np.abs(a).max()) for a, b in zip(outs[0], outs[1])]
    # the fma path stores roped K pairs in its slot order (rope_slot): bring
    # the scalar path's rows into the same order before comparing bytes
    half = cfg.head_dim // 2
    perm = np.arange(cfg.head_dim)
    for q in range(half):
        g8, j = q >> 3, q & 7
        if (g8 + 1) * 8 <= half:
            j = j + 2 if j in (2, 3) else j - 2 if j in (4, 5) else j
        o = g8 * 8 + j
        perm[2 * o], perm[2 * o + 1] = 2 * q, 2 * q + 1
    kvfrac = {}
    for layer in kvs[0]:
        (k0, v0), (k1, v1) = kvs[0][layer], kvs[1][layer]
        k1 = k1.reshape(-1, cfg.head_dim)[:, perm].reshape(-1)
        kvfrac[str(layer)] = float(max((k0 != k1).mean(), (v0 != v1).mean()))
    return {"logits_rel": logit, "kv_frac": kvfrac}


def main():
    ref = Reference("fma", 0)
    g = {"isa": "fma", "ops": run_ops(ref)}
    with open(os.path.join(OUT, "ops.json"), "w") as f:
        json.dump(g, f, indent=1, sort_keys=True)

    kat = {}
    hw = HostWeights.bind_test_kat()
    kat["bind_123"] = [int(x) for x in ref.generate(hw.desc, [1, 2, 3], 3, max_seq=8)]
    kat["bind_567"] = [int(x) for x in ref.generate(hw.desc, [5, 6, 7], 3, max_seq=8)]
    hs = HostWeights.shift_demo_kat()
    kat["shift_abcdefgh"] = [int(x) for x in ref.generate(hs.desc, list(range(97, 105)), 16, max_seq=1024)]
    with open(os.path.join(OUT, "kat.json"), "w") as f:
        json.dump(kat, f, indent=1)

    # synthetic generator + RoPE tables of every config (pins the host helpers)
    host = {"synth_q8": sha(synth_q8(1234, 5, 64, 512)), "synth_f32": sha(synth_f32(1234, 6, 4096)),
            "synth_ids": sha(synth_ids(1234, 7, 151936, 1000))}
    for key in ("c0", "c1", "c2", "c3"):
        c = CONFIGS[key]
        cs, sn = rope_table(c.max_seq, c.head_dim, c.theta)
        rc, rs = cs.copy(), sn.copy()
        ref.rope_table(c.max_seq, c.head_dim, C.c_float(c.theta), p(rc), p(rs))
        assert np.array_equal(cs, rc) and np.array_equal(sn, rs), key
        host[f"rope_{key}"] = sha(np.concatenate([cs, sn]))
    with open(os.path.join(OUT, "host.json"), "w") as f:
        json.dump(host, f, indent=1, sort_keys=True)

    # the 128-token greedy sequence + teacher-forced logits
    c0 = CONFIGS["c0"]
    hw0 = HostWeights.synthetic(c0)
    pr = prompt_ids(c0)
    ids = ref.generate(hw0.desc, pr, c0.new_tokens, max_seq=c0.max_seq)
    rows, kv = teacher_forced(ref, hw0, pr, 16)
    # the reference's sampler and repetition penalty (generate.h:50-77)
    sampled = ref.generate(hw0.desc, pr, 64, temperature=0.8, rep=1.3, max_seq=c0.max_seq)
    penalized = ref.generate(hw0.desc, pr, 64, temperature=0.0, rep=1.3, max_seq=c0.max_seq)
    with open(os.path.join(OUT, "c0.json"), "w") as f:
        json.dump({"seed": 1234, "prompt": [int(x) for x in pr], "greedy": [int(x) for x in ids],
                   "sampled_t0.8_p1.3": [int(x) for x in sampled],
                   "greedy_p1.3": [int(x) for x in penalized],
                   "teacher_forced": rows, "kv_sha": kv, "isa_spread": isa_spread(hw0, pr, 16)}, f, indent=1)

    # configs[1] shape: short prompt (the CPU prefill path is scalar), 16 tokens
    c1 = CONFIGS["c1"]
    hw1 = HostWeights.synthetic(c1)
    pr1 = prompt_ids(c1, n=16)
    ids1 = ref.generate(hw1.desc, pr1, 16, max_seq=c1.max_seq)
    rows1, kv1 = teacher_forced(ref, hw1, pr1, 4)
    with open(os.path.join(OUT, "c1.json"), "w") as f:
        json.dump({"seed": 1234, "prompt": [int(x) for x in pr1], "greedy": [int(x) for x in ids1],
                   "teacher_forced": rows1, "kv_sha": kv1, "isa_spread": isa_spread(hw1, pr1, 4)}, f, indent=1)

    # configs[2] shape, Q8_0 and fp32 variants, max context 256: 8-token prompt + 3 steps
    from dataclasses import replace
    c2 = {}
    for key in ("c2", "c2f"):
        cfg = replace(CONFIGS[key], max_seq=256)
        hw2 = HostWeights.synthetic(cfg)
        c2[key] = {"isa_spread": isa_spread(hw2, prompt_ids(cfg, n=8), 3)}
    with open(os.path.join(OUT, "c2.json"), "w") as f:
        json.dump(c2, f, indent=1)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
