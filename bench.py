#!/usr/bin/env python
"""Benchmark of the B200 decode path (driver contract: one JSON line on rank 0).

Headline workload (default): BASELINE.json configs[3], the Llama-3-8B shape
with synthetic seeded Q8_0 weights (7.98 GB per token, far above the 126 MB
L2): a 4096-token random prompt is prefilled, then one bench step = rewind to
that context and decode 64 greedy batch-1 tokens (positions 4097..4160).
Metric: decode tokens/s (CUDA events on the launching stream, max over
ranks), with the decode kernel's HBM roofline, the 4096-token prefill tok/s,
the end-to-end numbers through the public calls with host buffers, and the
reference's own CPU decode at the same context timed on this host.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 (torchrun): tensor parallel over the N ranks (QKV / gate-up column
split, O / down row split, the decode kernel's own NVLink exchange of the
partial sums; prefill with NCCL all-reduces), value = tokens / max-over-ranks
time, "scaling": "strong"; rank 0 also checks its tokens against the whole
model on one GPU. --impl reference times the reference (oracle/_ref) on the
host cores, on rank 0 only.

Other workloads (not the driver's line): --workload c1 (configs[1] decode),
c4 (configs[4] batched decode sweep), prefill (--model c1/c2/c3), kquant.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s"
UNIT = "tok/s"
PROMPT = 512            # --workload c1: prompt and decode tokens per step
DECODE = 256
HEAD_CFG = "c3"         # the headline: configs[3] at context CTX
CTX = 4096
HEAD_MAX_SEQ = 4352
DECODE_C3 = 64          # decode tokens per step of the headline
E2E_NEW = 128           # new tokens of one end-to-end call
REF_TOKENS_PER_STEP = 2  # reference arm: decode tokens of its bounded sample per step
KCLASSES = ["embed", "qkv_gemv", "rope_quant", "attention", "o_proj_gemv", "gate_up_gemv",
            "down_gemv", "lm_head_gemv_argmax"]


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index):
        self.dev = dev_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "samples": len(sm),
                "reasons": sorted(reasons)}


def reference_decode_sample(hw, threads, new_tokens=16, prompt_len=16, reps=2):
    """The reference's own generate() (oracle/_ref: the jieyu headers compiled
    unmodified) on this host: decode tok/s over a bounded sample."""
    import numpy as np

    from jieyu_b200.model import prompt_ids
    from oracle.bind import Reference
    ref = Reference("fma", threads)
    pr = prompt_ids(hw.cfg, n=prompt_len)
    dec_tok, dec_s, tot_s = 0, 0.0, 0.0
    times = np.zeros(3)
    for _ in range(reps):
        out = ref.generate(hw.desc, pr, new_tokens, max_seq=hw.cfg.max_seq, times=times)
        n_new = len(out) - prompt_len
        dec_tok += n_new - 1          # first token comes from the prefill pass
        dec_s += times[1]
        tot_s += times[2]
    return dec_tok / dec_s, (reps * new_tokens) / tot_s, ref.lib.jyref_threads()


class RefContextDecode:
    """The reference's decode at context CTX, timed on this host's cores:
    oracle/_ref (the jieyu headers compiled unmodified) runs generate_cached's
    step body (embedding row, forward_cached, LM head, greedy pick;
    generate.h:40-60) from a KV cache holding a seeded context of `ctx`
    positions (oracle.synth.context_kv), i.e. the decode work of position
    ctx, ctx + 1, ... without the CPU prefill of the prompt (hours at the
    8B shape on the scalar m>1 path). `desc` is any jyc_model_desc-layout
    ctypes structure over host weights."""

    def __init__(self, desc, layers, kv_heads, head_dim, max_seq, ctx, threads):
        from oracle import synth
        from oracle.bind import Reference
        self.ref = Reference("fma", threads)
        self.desc, self.ctx = desc, ctx
        self.cache = self.ref.cache_create(layers, max_seq, kv_heads, head_dim)
        for l, k, ks, v, vs in synth.context_kv(layers, ctx, kv_heads, head_dim):
            self.ref.cache_write(self.cache, l, ctx, k.ctypes.data, ks.ctypes.data, v.ctypes.data, vs.ctypes.data)
        self.cores = self.ref.lib.jyref_threads()

    def run(self, n: int):
        """n greedy decode tokens from position ctx; returns seconds per token."""
        _, t = self.ref.decode_steps(self.desc, self.cache, self.ctx, 1, n)
        return t

    def close(self):
        if self.cache:
            self.ref.cache_free(self.cache)
            self.cache = None


def head_config():
    """The headline's config keys (shared by both arms)."""
    return {"workload": f"configs[3] Llama-3-8B shape (Q8_0 weights N(0, 0.02), seeded): batch-1 greedy decode "
                        f"at context {CTX} ({DECODE_C3} tokens per step after a {CTX}-token random prompt)",
            "model": "c3_llama3_8b", "global_batch": 1, "seq_len": CTX + 1 + DECODE_C3,
            "l2": "inputs larger than L2 (7.98 GB of weights per token / N ranks vs 126 MB L2)"}


def run_reference_arm(args):
    """The reference arm: the reference's own CPU decode (oracle/_ref) of the
    headline workload (configs[3] shape, Q8_0, context 4096) on this host's
    cores, a bounded sample per step (REF_TOKENS_PER_STEP decode tokens).
    The seeded weights come from liboracle.so's generator (oracle.synth),
    byte-identical to the GPU arm's: the product library is not loaded."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    from oracle import synth
    from oracle.bind import reference_available
    if not reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libjyref.so was not built"}))
        return 0
    shape = synth.SHAPES[HEAD_CFG]
    threads = os.cpu_count() or 1
    sm = synth.SynthModel(shape, HEAD_MAX_SEQ)
    rd = RefContextDecode(sm.desc, shape.layers, shape.kv_heads, shape.head_dim, HEAD_MAX_SEQ, CTX, threads)
    for _ in range(args.warmup):
        rd.run(1)
    toks, secs = 0, 0.0
    t0 = time.time()
    for _ in range(args.steps):
        t = rd.run(REF_TOKENS_PER_STEP)
        toks += len(t)
        secs += float(t.sum())
    wall = time.time() - t0
    value = toks / secs
    rd.close()
    sample = (f"jieyu reference (oracle/_ref: the unmodified headers, JIEYU_ISA=fma, OpenMP, {rd.cores} threads) "
              f"decoding configs[3]-shaped seeded Q8_0 weights at context {CTX} (a seeded int8 K/V context "
              f"written into its __KVcache; generate_cached's step body per token), {REF_TOKENS_PER_STEP} "
              f"tokens per step; value = decode tokens / their seconds")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": dict(head_config(), parallelism="host threads"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": rd.cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_c1(args):
    import numpy as np
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    lib = _capi.load()
    cfg = CONFIGS["c1"]
    hw = HostWeights.synthetic(cfg)
    m = DeviceModel(hw)
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    prompt = torch.from_numpy(prompt_ids(cfg)).cuda()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    with torch.cuda.stream(stream):
        # prefill once (KV of positions 0..511 stays resident), then timed prefills
        m.prefill_device(prompt.data_ptr(), PROMPT, s)
        stream.synchronize()
        pf_ms = []
        for _ in range(2):
            a, b = ev(), ev()
            a.record(stream)
            m.prefill_device(prompt.data_ptr(), PROMPT, s)
            b.record(stream)
            stream.synchronize()
            pf_ms.append(a.elapsed_time(b))
        prefill_tps = PROMPT / (min(pf_ms) / 1e3)

        def step():
            m.rewind(PROMPT + 1, s)   # prompt + the prefill's token; KV 0..512 resident
            m.decode_device(DECODE, s)

        for _ in range(args.warmup):
            step()
        stream.synchronize()
        barrier()
        sampler = ClockSampler(local)
        sampler.start()
        launches0 = lib.jyc_kernel_launches()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = ev(), ev()
        if args.nvtx:
            torch.cuda.nvtx.range_push("timed")
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        stream.synchronize()
        if args.nvtx:
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
        launches = lib.jyc_kernel_launches() - launches0
        clocks = sampler.stop()
        ms_local = e0.elapsed_time(e1)
        assert m.length(s) == PROMPT + 1 + DECODE, "decode did not run every step"
        ms = max_over_ranks(ms_local)
        tokens = sum_over_ranks(args.steps * DECODE)
        value = tokens / (ms / 1e3)
        ms_per_step = ms / args.steps

        # per-kernel device time of the decode step (event after every kernel)
        m.rewind(PROMPT + 1, s)
        kms = (C.c_double * 8)()
        kl = (C.c_int * 8)()
        kb = (C.c_double * 8)()
        _capi.check(lib.jyc_model_profile_decode(m.h, 64, s, kms, kl, kb))
        stream.synchronize()

    # roofline of the dominant kernel (HBM-bound): the decode megakernel (one
    # launch per token, algorithmic bytes = weights + KV read per token), or on
    # the generic path the largest kernel class
    peak, peak_kind = measured_peaks()
    mega = lib.jyc_model_decode_path(m.h) == 2
    classes = ["mega_step_kernel"] + [f"unused{i}" for i in range(1, 8)] if mega else KCLASSES
    shares = {classes[i]: kms[i] for i in range(8) if kl[i] > 0}
    total_k = sum(shares.values())
    dom = max(range(8), key=lambda i: kms[i])
    per_launch_ms = kms[dom] / max(kl[dom], 1)
    achieved = kb[dom] / (per_launch_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic_c1_decode.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get(classes[dom])
    weight_bytes = hw.weight_bytes_per_token()
    kv_bytes = float(lib.jyc_model_kv_bytes_per_token(m.h, PROMPT + 1 + DECODE // 2))
    step_gbs = (weight_bytes + kv_bytes) / (ms_per_step / DECODE / 1e3) / 1e9

    # end to end through the C ABI (jyc_generate) with host buffers
    pin_prompt = torch.from_numpy(prompt_ids(cfg)).pin_memory()
    pin_out = torch.zeros(cfg.max_seq + 1, dtype=torch.int32).pin_memory()
    e = np.zeros(1, np.int32)
    cb = _capi.TOKEN_CB()
    def gen():
        n = lib.jyc_generate(m.h, pin_prompt.data_ptr(), PROMPT, e.ctypes.data, 0, DECODE, 0.0,
                             pin_out.data_ptr(), 1.0, cb, None)
        return _capi.check(n)
    gen()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    e2e_steps = max(1, min(args.steps, 3))
    for _ in range(e2e_steps):
        n = gen()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    assert n == PROMPT + DECODE
    e2e_value = sum_over_ranks(e2e_steps * DECODE) / e2e_s

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        dec, _, cores = reference_decode_sample(hw, threads)
        cpu = {"value": dec, "unit": UNIT, "cores": cores, "kind": "reference",
               "sample": "jieyu reference generate() (oracle/_ref, unmodified headers, "
                         "JIEYU_ISA=fma) on the configs[1] weights, 16-token prompt + 16 greedy "
                         "tokens, x2; decode tok/s first->last token"}

    m.close()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[1] Qwen2.5-0.5B shape (Q8_0, tied embedding, QKV bias): "
                               "256 greedy decode tokens after a 512-token prompt, batch 1",
                   "model": cfg.name, "global_batch": world, "seq_len": PROMPT + DECODE,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (525 MB of weights per token vs 126 MB L2)"},
        "hbm": {"gbs_per_step": step_gbs, "bytes_per_token": weight_bytes + kv_bytes,
                "frac_of_peak": step_gbs / peak, "peak_gbs": peak, "peak_kind": peak_kind},
        "roofline": {"bound": "hbm", "kernel": classes[dom], "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "bytes_per_launch": kb[dom], "launch_ms": per_launch_ms,
                     "peak_kind": peak_kind},
        "kernel_ms_per_token": {k: v / 64 for k, v in shares.items()},
        "kernel_share": {k: (v / total_k if total_k else None) for k, v in shares.items()},
        "prefill": {"value": prefill_tps, "unit": "tok/s", "prompt": PROMPT},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": PROMPT * 4,
                "d2h_bytes_per_step": DECODE * 4 + 96,
                "note": "jyc_generate from pinned host ids: H2D prompt, prefill, 256 decode "
                        "steps, D2H of the new ids; new tokens / wall time"},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def traffic_capture(kernel_src: str, key: str):
    """DRAM bytes per launch of the decode kernel from a stored ncu capture
    (profiles/traffic_decode.json), used only while the kernel source it was
    taken on is unchanged (sha256 of mega.cu); else None."""
    import hashlib
    path = os.path.join(ROOT, "profiles", "traffic_decode.json")
    if not os.path.exists(path):
        return None, "no stored capture"
    with open(path) as f:
        d = json.load(f)
    with open(kernel_src, "rb") as f:
        sha = hashlib.sha256(f.read()).hexdigest()[:16]
    e = d.get(key)
    if not e:
        return None, f"no stored capture for {key}"
    if e.get("mega_cu_sha16") != sha:
        return None, f"stored capture is of another kernel source ({e.get('mega_cu_sha16')} != {sha})"
    return float(e["bytes_per_launch"]), e.get("how", "")


def run_headline(args):
    """The headline line: configs[3] (Llama-3-8B shape, Q8_0) batch-1 greedy
    decode at context 4096. One step = rewind to the 4096-token prompt + its
    first token and decode DECODE_C3 tokens (positions 4097..). N = 1: the
    whole model on one GPU, one decode-kernel launch per token. N > 1
    (torchrun): tensor parallel over the N ranks (jieyu_b200.tp.TPDecoder,
    the kernel's own NVLink exchange of the O / down partials), value = tokens
    / max-over-ranks time ("scaling": "strong": the same model whatever N).
    The same line carries the 4096-token prefill (tensor parallel at N > 1),
    the end-to-end numbers through the public calls with host buffers, the
    roofline of the decode kernel and, at N > 1, a check of rank 0's tokens
    against the whole model on one GPU."""
    import numpy as np
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids, with_max_seq

    world, rank, local = env_int("WORLD_SIZE", 1), env_int("RANK", 0), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = _capi.load()
    cfg = with_max_seq(CONFIGS[HEAD_CFG], HEAD_MAX_SEQ)
    hw = HostWeights.synthetic(cfg)
    prompt = prompt_ids(cfg, n=CTX)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    if world == 1:
        m = DeviceModel(hw)
        h = m.h
        stream = torch.cuda.Stream()
        ids = torch.from_numpy(prompt).cuda()

        def prefill():
            m.prefill_device(ids.data_ptr(), CTX, stream.cuda_stream)

        def step():
            m.rewind(CTX + 1, stream.cuda_stream)
            m.decode_device(DECODE_C3, stream.cuda_stream)
        parallelism = "single GPU"
    else:
        from jieyu_b200.tp import TPDecoder
        tp = TPDecoder(hw, rank, world, mode="kernel")
        h = tp.m.h
        stream = tp.stream

        def prefill():
            tp.prefill(prompt)

        def step():
            _capi.check(lib.jyc_model_rewind(tp.m.h, CTX + 1, stream.cuda_stream))
            tp.step(DECODE_C3)
        parallelism = f"tp{world}"
    s = stream.cuda_stream

    # prefill of the 4096-token prompt (KV of positions 0..4095 stays resident)
    with torch.cuda.stream(stream):
        prefill()
        stream.synchronize()
        barrier()
        pf_ms = []
        for _ in range(2):
            a, b = ev(), ev()
            a.record(stream)
            prefill()
            b.record(stream)
            stream.synchronize()
            pf_ms.append(a.elapsed_time(b))
        pf_ms = max_over_ranks(min(pf_ms))
        first_tokens = None
        for i in range(args.warmup):
            step()
            if i == 0:
                stream.synchronize()
                n_tok = CTX + 1 + DECODE_C3
                dev_toks = torch.as_tensor(_DevBuf(lib.jyc_model_tokens_device(h), n_tok), device="cuda")
                first_tokens = dev_toks[CTX:n_tok].cpu().numpy().copy()
        stream.synchronize()
        barrier()
        sampler = ClockSampler(local)
        sampler.start()
        launches0 = lib.jyc_kernel_launches()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = ev(), ev()
        if args.nvtx:
            torch.cuda.nvtx.range_push("timed")
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        stream.synchronize()
        if args.nvtx:
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
        launches = lib.jyc_kernel_launches() - launches0
        clocks = sampler.stop()
    assert lib.jyc_device_error(1) == 0, "a bounded wait of the decode kernel gave up"
    ms = max_over_ranks(e0.elapsed_time(e1))
    tokens = args.steps * DECODE_C3
    value = tokens / (ms / 1e3)
    ms_tok = ms / tokens

    # roofline of the decode kernel (one launch per token): algorithmic bytes
    # of one launch on this rank (its weights + the KV rows it reads at the
    # mean context of a step) over the event-timed time per launch
    peak, peak_kind = measured_peaks()
    w_rank = float(lib.jyc_model_weight_bytes_per_token(h))
    kv_rank = float(lib.jyc_model_kv_bytes_per_token(h, CTX + 1 + DECODE_C3 // 2))
    bytes_launch = w_rank + kv_rank
    achieved = bytes_launch / (ms_tok / 1e3) / 1e9
    traffic, traffic_note = traffic_capture(os.path.join(ROOT, "jieyu_b200", "csrc", "mega.cu"),
                                            f"{HEAD_CFG}_tp{world}")

    # end to end through the public calls with host buffers: the prompt from
    # pinned host memory, the 4096-token prefill, DECODE_C3 new tokens read
    # back to the host in blocks (jyc_generate with a token callback at N = 1,
    # TPDecoder.generate at N > 1); decode tok/s first -> last token as the
    # reference's -tokenspeed splits it (pipeline.h:356-367), and the whole call
    e2e_n = E2E_NEW
    stamps = []

    def cb(tok):
        stamps.append(time.perf_counter())
        return False
    pin_prompt = torch.from_numpy(prompt).pin_memory()
    e2e_runs = []
    for _ in range(2):
        stamps.clear()
        barrier()
        t0 = time.perf_counter()
        if world == 1:
            got = m.generate(pin_prompt.numpy(), e2e_n, cb=cb)
        else:
            got = tp.generate(pin_prompt.numpy(), e2e_n, cb=cb)
        t1 = time.perf_counter()
        assert len(got) == CTX + e2e_n
        e2e_runs.append((t1 - t0, stamps[0] - t0, stamps[-1] - stamps[0]))
    whole, to_first, first_last = e2e_runs[-1]
    whole = max_over_ranks(whole)
    to_first = max_over_ranks(to_first)
    first_last = max_over_ranks(first_last)
    e2e_decode = (e2e_n - 1) / first_last

    # N > 1: rank 0's tokens against the whole model on one GPU
    tp_check = None
    if world > 1:
        tp.close()
        barrier()
        if rank == 0:
            m1 = DeviceModel(hw)
            one = m1.generate(prompt, DECODE_C3 + 1)[CTX:CTX + DECODE_C3 + 1]
            same = int(np.argmax(one != first_tokens)) if not np.array_equal(one, first_tokens) else None
            tp_check = {"tokens": int(DECODE_C3 + 1), "identical": same is None, "first_difference": same}
            if same is not None:  # the top-2 gap of the whole model's logits at that step
                lg = m1.forward_logits(np.array([one[same - 1] if same else prompt[-1]], np.int32),
                                       CTX + same - 1)
                top = np.sort(lg.astype(np.float64))[-2:]
                tp_check["top2_gap_rel"] = float((top[1] - top[0]) / np.abs(lg).max())
            m1.close()
    else:
        m.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rd = RefContextDecode(hw.desc, cfg.layers, cfg.kv_heads, cfg.head_dim, cfg.max_seq, CTX,
                              os.cpu_count() or 1)
        rd.run(1)
        t = rd.run(REF_TOKENS_PER_STEP)
        rd.close()
        cpu = {"value": len(t) / float(t.sum()), "unit": UNIT, "cores": rd.cores, "kind": "reference",
               "sample": f"jieyu reference (oracle/_ref, unmodified headers, JIEYU_ISA=fma) decoding "
                         f"{REF_TOKENS_PER_STEP} tokens at context {CTX} on the same configs[3] weights "
                         f"(seeded int8 K/V context in its __KVcache; generate_cached's step body)"}
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(head_config(), parallelism=parallelism),
        "ms_per_token": ms_tok,
        "hbm_per_gpu": {"bytes_per_token": bytes_launch, "gbs": achieved, "frac_of_peak": achieved / peak,
                        "peak_gbs": peak, "peak_kind": peak_kind},
        "roofline": {"bound": "hbm", "kernel": "mega_step_kernel", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_note,
                     "bytes_per_launch": bytes_launch, "launch_ms": ms_tok, "peak_kind": peak_kind},
        "prefill": {"value": CTX / (pf_ms / 1e3), "unit": "tok/s", "prompt": CTX, "ms": pf_ms,
                    "parallelism": parallelism},
        "e2e": {"value": e2e_decode, "unit": UNIT, "h2d_bytes_per_step": CTX * 4,
                "d2h_bytes_per_step": e2e_n * 4,
                "whole_call_s": whole, "whole_call_new_tok_s": e2e_n / whole, "prefill_s": to_first,
                "note": f"{'jyc_generate' if world == 1 else 'TPDecoder.generate'}: {CTX} prompt ids from pinned "
                        f"host memory, prefill, {e2e_n} greedy tokens read back to the host in blocks of "
                        f"1..32 (token callback); value = decode tokens/s first -> last new token, as the "
                        f"reference's -tokenspeed; whole_call includes the prefill"},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if tp_check is not None:
        line["tp_check"] = tp_check
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


class _DevBuf:
    """A device buffer of the library seen by torch (zero copy)."""

    def __init__(self, ptr: int, n: int, typestr: str = "<i4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def run_c4(args):
    """batched decode sweep on the Llama-3.2-1B shape (Q8_0), one
    GPU. B = 1, 4, 16, 32, 64 sequences, each prefilled with its own
    2048-token random prompt; one step = rewind every sequence to context
    2049 and decode 128 greedy tokens per sequence. B = 1 runs the
    single-sequence decode kernel, B = 2..8 the few-row matmul (CUDA
    cores), B >= 9 the tcgen05 tiles. Also times
    the 2048-token prefill (configs[2]'s prefill)."""
    import numpy as np
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS, BatchDecoder, DeviceModel, HostWeights, synth_ids

    if env_int("RANK", 0) != 0:
        return 0
    torch.cuda.set_device(env_int("LOCAL_RANK", 0))
    cfg = CONFIGS["c4"]
    ctx, new = 2048, args.decode_tokens
    hw = HostWeights.synthetic(cfg)
    m = DeviceModel(hw)
    lib = _capi.load()
    peak, peak_kind = measured_peaks()
    tpeak = 1590.0  # the fallback burst bf16 figure when the driver's file is absent
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            tpeak = float(json.load(f).get("bf16_tflops", tpeak))
    w_bytes = float(lib.jyc_model_weight_bytes_per_token(m.h))
    # multiply-adds per token of the matmuls (Q, K, V, O, gate, up, down; LM head)
    D, F, qd, kvd = cfg.hidden, cfg.inter, cfg.q_dim, cfg.kv_dim
    macs = cfg.layers * (D * (qd + 2 * kvd) + qd * D + 2 * D * F + F * D) + cfg.vocab * D
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    prompts = [synth_ids(2026, 4000 + b, cfg.vocab, ctx) for b in range(64)]
    sweep = []
    prefill_tps = None
    clocks = ClockSampler(env_int("LOCAL_RANK", 0))
    clocks.start()
    for B in [int(x) for x in args.seqs.split(",")]:
        bt = None
        if B == 1:
            ids = torch.from_numpy(prompts[0]).cuda()
            with torch.cuda.stream(stream):
                e0, e1 = ev(), ev()
                m.prefill_device(ids.data_ptr(), ctx, s)  # warm
                e0.record(stream)
                m.prefill_device(ids.data_ptr(), ctx, s)
                e1.record(stream)
                stream.synchronize()
                prefill_tps = ctx / (e0.elapsed_time(e1) / 1e3)

            def step():
                m.rewind(ctx + 1, s)
                m.decode_device(new, s)
            path = "single-sequence decode kernel"
        else:
            bt = BatchDecoder(m, B)
            for b in range(B):
                bt.prefill(b, prompts[b])

            def step(bt=bt):
                bt.rewind(ctx + 1, s)
                bt.decode(new, s)
            path = "tcgen05 tiles" if bt.path() == 2 else "few-row matmul"
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step()
            stream.synchronize()
            if args.nvtx:
                torch.cuda.nvtx.range_push("timed")
            e0, e1 = ev(), ev()
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
            stream.synchronize()
            if args.nvtx:
                torch.cuda.nvtx.range_pop()
        ms = e0.elapsed_time(e1) / args.steps / new  # per batched step
        kv = B * float(lib.jyc_model_kv_bytes_per_token(m.h, ctx + new // 2))
        gbs = (w_bytes + kv) / (ms / 1e3) / 1e9
        tflops = 2.0 * macs * B / (ms / 1e3) / 1e12
        sweep.append({"seqs": B, "tok_s": B / (ms / 1e3), "ms_per_step": ms, "path": path,
                      "hbm_gbs": gbs, "hbm_frac": gbs / peak, "bytes_per_step": w_bytes + kv,
                      "tensor_tflops": tflops, "tensor_frac": tflops / tpeak})
        assert lib.jyc_device_error(1) == 0
        if bt is not None:
            bt.close()
    clk = clocks.stop()
    m.close()
    best = max(sweep, key=lambda r: r["tok_s"])
    line = {
        "metric": "batched decode aggregate tok/s (configs[4])", "value": sweep[-1]["tok_s"], "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"configs[4] Llama-3.2-1B shape, Q8_0, {ctx}-token context per sequence, "
                               f"{new} greedy tokens per sequence per step",
                   "l2": "inputs larger than L2 (1.3 GB of weights per step)"},
        "sweep": sweep, "best": {"seqs": best["seqs"], "tok_s": best["tok_s"]},
        "prefill": {"value": prefill_tps, "unit": "tok/s", "prompt": ctx, "model": "configs[2] shape (Q8_0)"},
        "peaks": {"hbm_gbs": peak, "hbm_kind": peak_kind, "bf16_tflops": tpeak,
                  "note": "tensor_tflops counts 2*params*seqs per step (the fp16 hi/lo split does 3x that)"},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_kquant(args):
    """K-quant weights (the formats of the reference's published downloads):
    one step = one m=1 matmul (jyc_matmul_qk) over every linear weight of the
    configs[2] shape (Llama-3.2-1B: 16 layers x Q, K, V, O, gate, up, down;
    0.55 / 0.67 / 0.80 GB per step for Q4_K / Q5_K / Q6_K, larger than L2),
    captured in one CUDA graph per format,
    seeded random blocks with finite scales. value = Q4_K weight GB/s; the
    roofline is HBM (algorithmic bytes = the blocks). The CPU baseline is the
    reference's own qmat::matmul_q on one layer's Q4_K matrices (oracle/_ref,
    else the oracle port), all host threads. The line also carries the
    decode tok/s of a configs[2]-shaped model in mixed K-quant formats
    (model_decode: the model path, the layer matrices read in place as
    K-quant blocks; beside it the same model with every matrix dequantised to
    fp32 at upload)."""
    import numpy as np
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS

    if env_int("RANK", 0) != 0:
        return 0
    torch.cuda.set_device(env_int("LOCAL_RANK", 0))
    cfg = CONFIGS["c2"]
    D, F, qd, kvd = cfg.hidden, cfg.inter, cfg.q_dim, cfg.kv_dim
    shapes = [(qd, D), (kvd, D), (kvd, D), (D, qd), (F, D), (F, D), (D, F)] * cfg.layers
    lib = _capi.load()
    peak, peak_kind = measured_peaks()
    stream = torch.cuda.Stream()
    x = torch.randn(max(D, F, qd), device="cuda", dtype=torch.float32)
    y = torch.empty(max(D, F, qd), device="cuda", dtype=torch.float32)
    bb = {0: 144, 1: 176, 2: 210}
    names = {0: "q4_K", 1: "q5_K", 2: "q6_K"}
    sweep = []
    clocks = ClockSampler(env_int("LOCAL_RANK", 0))
    clocks.start()
    for qt in (0, 1, 2):
        mats = []
        for (n, k) in shapes:
            w = torch.randint(0, 256, (n * (k // 256), bb[qt]), dtype=torch.uint8, device="cuda")
            if qt == 2:
                w[:, 208:210] = torch.tensor([0x00, 0x18], dtype=torch.uint8, device="cuda")  # fp16 2^-9
            else:
                w[:, 0:4] = torch.tensor([0x00, 0x18, 0x00, 0x14], dtype=torch.uint8, device="cuda")
            mats.append((w, n, k))
        nbytes = float(sum(w.numel() for w, _, _ in mats))

        def launch_all():
            for w, n, k in mats:
                _capi.check(lib.jyc_matmul_qk(x.data_ptr(), w.data_ptr(), y.data_ptr(), 1, n, k, qt,
                                              torch.cuda.current_stream().cuda_stream))
        with torch.cuda.stream(stream):
            launch_all()  # warm (module load)
            stream.synchronize()
        graph = torch.cuda.CUDAGraph()  # one step = one replay: no host launch gaps in the timing
        with torch.cuda.graph(graph, stream=stream):
            launch_all()
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                graph.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            stream.synchronize()
        del graph
        ms = e0.elapsed_time(e1) / args.steps
        gbs = nbytes / (ms / 1e3) / 1e9
        sweep.append({"format": names[qt], "ms_per_step": ms, "bytes_per_step": nbytes, "gbs": gbs,
                      "hbm_frac": gbs / peak, "launches_per_step": len(mats)})
        del mats
    # the model path: a configs[2]-shaped model in mixed K-quant formats
    # (HostWeights.synthetic_kquant), dequantised to fp32 once at upload,
    # greedy decode on the generic kernels after a 128-token prompt
    from jieyu_b200.model import DeviceModel, HostWeights, prompt_ids
    khw = HostWeights.synthetic_kquant(cfg)
    km = DeviceModel(khw)
    kids = torch.from_numpy(prompt_ids(cfg, n=128)).cuda()
    new = 64
    with torch.cuda.stream(stream):
        s = stream.cuda_stream
        km.prefill_device(kids.data_ptr(), 128, s)
        km.decode_device(8, s)  # warm (graph capture)
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        km.rewind(129, s)
        e0.record(stream)
        km.decode_device(new, s)
        e1.record(stream)
        stream.synchronize()
    kms = e0.elapsed_time(e1) / new
    kbytes = float(lib.jyc_model_weight_bytes_per_token(km.h))
    assert lib.jyc_device_error(1) == 0
    km.close()
    # the same model with every matrix dequantised to fp32 at upload (the
    # comparison path, JYC_KQ_FP32=1)
    os.environ["JYC_KQ_FP32"] = "1"
    try:
        km = DeviceModel(khw)
    finally:
        del os.environ["JYC_KQ_FP32"]
    with torch.cuda.stream(stream):
        s = stream.cuda_stream
        km.prefill_device(kids.data_ptr(), 128, s)
        km.decode_device(8, s)
        stream.synchronize()
        km.rewind(129, s)
        e0.record(stream)
        km.decode_device(new, s)
        e1.record(stream)
        stream.synchronize()
    fms = e0.elapsed_time(e1) / new
    fbytes = float(lib.jyc_model_weight_bytes_per_token(km.h))
    assert lib.jyc_device_error(1) == 0
    km.close()
    del khw
    model_line = {"tok_s": 1e3 / kms, "ms_per_token": kms, "bytes_per_token": kbytes,
                  "hbm_gbs": kbytes / (kms / 1e3) / 1e9, "hbm_frac": kbytes / (kms / 1e3) / 1e9 / peak,
                  "fp32_path": {"tok_s": 1e3 / fms, "ms_per_token": fms, "bytes_per_token": fbytes},
                  "note": "layer matrices read as K-quant blocks in place by the K-quant matmul, LM head "
                          "dequantised to fp32 at upload; fp32_path: every matrix dequantised to fp32 "
                          "(4 B per weight)"}
    clk = clocks.stop()
    # CPU baseline: the reference's matmul_q over one layer's Q4_K matrices
    rng = np.random.default_rng(7)
    host = []
    for (n, k) in shapes[:7]:
        b = rng.integers(0, 256, size=(n * (k // 256), 144), dtype=np.uint8)
        b[:, 0:4] = np.array([0x00, 0x18, 0x00, 0x14], np.uint8)
        host.append((np.ascontiguousarray(b), n, k))
    xa = np.random.default_rng(8).standard_normal(max(D, F)).astype(np.float32)
    ya = np.empty(max(D, F, qd), np.float32)
    cpu = None
    try:
        sys.path.insert(0, ROOT)
        from oracle.bind import Oracle, Reference, reference_available
        if reference_available():
            ref, kind = Reference(), "reference"
            fn = ref.lib.jyref_matmul_qk
        else:
            ref, kind = Oracle(), "port"
            fn = ref.lib.jyo_matmul_qk
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 3.0:
            for b, n, k in host:
                fn(xa.ctypes.data, b.ctypes.data, ya.ctypes.data, 1, n, k, 0)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        lbytes = float(sum(b.nbytes for b, _, _ in host))
        cpu = {"value": lbytes / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": kind,
               "sample": f"one configs[2] layer's 7 Q4_K matrices ({lbytes / 1e6:.1f} MB), m=1, {reps} passes"}
    except Exception as e:  # the checker is absent on this host: report why
        cpu = {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port", "sample": f"unavailable: {e}"}
    q4 = sweep[0]
    line = {
        "metric": "K-quant matmul weight GB/s (configs[2] shape, m=1)", "value": q4["gbs"], "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "jyc_matmul_qk over the 112 linear weights of the configs[2] shape, one activation row",
                   "l2": "inputs larger than L2 (0.55 GB of Q4_K blocks per step)"},
        "sweep": sweep, "model_decode": model_line,
        "roofline": {"bound": "hbm", "kernel": "kq_gemv_smem_kernel<Q4_K, 1>", "achieved": q4["gbs"], "peak": peak,
                     "unit": "GB/s", "frac": q4["gbs"] / peak, "traffic": None, "peak_kind": peak_kind},
        "gpu_launches": len(shapes) * args.steps, "clocks": clk, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_prefill(args):
    """Prompt prefill of one config (the BASELINE metric's prefill tok/s):
    configs[1] 512 tokens, configs[2] 2048, configs[3] 4096, random seeded
    ids; one step = one whole prefill (K/V of every position written, first
    token picked). One GPU: the batched prefill. N GPUs (torchrun, configs[3]):
    tensor parallel (jieyu_b200.tp.TPDecoder.prefill: shards' O and down
    partials all-reduced over NCCL, one prompt per step over all ranks:
    "scaling": "strong"), max over ranks. Roofline: the tensor pipe;
    algorithmic FLOPs = 2 x matmul parameters x tokens + causal attention
    4 L H hd T(T+1)/2."""
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids

    world, rank, local = env_int("WORLD_SIZE", 1), env_int("RANK", 0), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    cfg = CONFIGS[args.model]
    T = cfg.prompt_len
    hw = HostWeights.synthetic(cfg)
    lib = _capi.load()
    D, F, qd, kvd = cfg.hidden, cfg.inter, cfg.q_dim, cfg.kv_dim
    params = cfg.layers * (D * (qd + 2 * kvd) + qd * D + 3 * D * F)
    flops = 2.0 * params * T + 4.0 * cfg.layers * cfg.heads * cfg.head_dim * T * (T + 1) / 2
    tpeak = 1590.0
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            tpeak = float(json.load(f).get("bf16_tflops", tpeak))
    if world > 1:
        from jieyu_b200.tp import TPDecoder
        tp = TPDecoder(hw, rank, world, mode="kernel")
        prompt = prompt_ids(cfg, n=T)
        stream = tp.stream

        def step():
            tp.prefill(prompt)
        close = tp.close
    else:
        m = DeviceModel(hw)
        ids = torch.from_numpy(prompt_ids(cfg, n=T)).cuda()
        stream = torch.cuda.Stream()

        def step():
            m.prefill_device(ids.data_ptr(), T, stream.cuda_stream)
        close = m.close
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        clocks = ClockSampler(local)
        clocks.start()
        if args.nvtx:
            torch.cuda.nvtx.range_push("timed")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = lib.jyc_kernel_launches()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        stream.synchronize()
        if args.nvtx:
            torch.cuda.nvtx.range_pop()
        clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert lib.jyc_device_error(1) == 0
    launches = lib.jyc_kernel_launches() - l0
    close()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    tflops = flops / (ms / 1e3) / 1e12
    line = {
        "metric": f"prefill tok/s ({args.model})", "value": T / (ms / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: prefill of a {T}-token random prompt (Q8_0 weights)",
                   "parallelism": f"tp{world}" if world > 1 else "single GPU",
                   "l2": "weights larger than L2 (126 MB)"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": tpeak * world, "unit": "TFLOP/s",
                     "frac": tflops / (tpeak * world), "flops_per_step": flops,
                     "note": "algorithmic FLOPs over all GPUs; the exact fp16 hi/lo split issues 3x the matmul "
                             "MMA work"},
        "gpu_launches": int(launches), "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_c2(args):
    """configs[2] (Llama-3.2-1B shape, Q8_0 and fp32 weights, one GPU): batch-1
    greedy decode at KV contexts of 1024, 4096 and 16384 positions, and the
    prefill of a 2048-token random prompt. The context is a seeded int8 K/V
    cache written into the device cache (oracle.synth.context_kv through
    jyc_model_write_kv; the decode step reads it exactly as it reads a
    prefilled one), then one step = rewind to ctx + 1 tokens and decode
    DECODE_C2 tokens. Per (weights, context): tok/s, the bytes one token
    reads (weights + the KV rows of its positions) and their HBM rate against
    the measured peak. value = the Q8_0 decode tok/s at context 4096."""
    import numpy as np
    import torch

    from jieyu_b200 import _capi
    from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids
    from oracle.synth import context_kv

    if env_int("RANK", 0) != 0:
        return 0
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    lib = _capi.load()
    peak, peak_kind = measured_peaks()
    DECODE_C2 = 64
    stream = torch.cuda.Stream()
    s = stream.cuda_stream
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    sweep, prefill = [], None
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = lib.jyc_kernel_launches()
    for key in ("c2", "c2f"):
        cfg = CONFIGS[key]
        hw = HostWeights.synthetic(cfg)
        m = DeviceModel(hw)
        w_bytes = float(lib.jyc_model_weight_bytes_per_token(m.h))
        if key == "c2":  # the 2048-token prefill (configs[2]'s prefill line)
            ids = torch.from_numpy(prompt_ids(cfg, n=2048)).cuda()
            with torch.cuda.stream(stream):
                m.prefill_device(ids.data_ptr(), 2048, s)
                a, b = ev(), ev()
                a.record(stream)
                m.prefill_device(ids.data_ptr(), 2048, s)
                b.record(stream)
                stream.synchronize()
            prefill = {"value": 2048 / (a.elapsed_time(b) / 1e3), "unit": "tok/s", "prompt": 2048,
                       "ms": a.elapsed_time(b)}
        tok = int(prompt_ids(cfg, n=1, index=7)[0])
        for ctx in (1024, 4096, 16384):
            for l, k, ks, v, vs in context_kv(cfg.layers, ctx, cfg.kv_heads, cfg.head_dim):
                m.write_kv(l, k, ks, v, vs)
            m.forward_logits(np.array([tok], np.int32), ctx)  # token at ctx, its KV row appended

            def step():
                m.rewind(ctx + 1, s)
                m.decode_device(DECODE_C2, s)
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    step()
                stream.synchronize()
                e0, e1 = ev(), ev()
                e0.record(stream)
                for _ in range(args.steps):
                    step()
                e1.record(stream)
                stream.synchronize()
            assert lib.jyc_device_error(1) == 0, "a bounded wait of the decode kernel gave up"
            ms_tok = e0.elapsed_time(e1) / (args.steps * DECODE_C2)
            kv = float(lib.jyc_model_kv_bytes_per_token(m.h, ctx + 1 + DECODE_C2 // 2))
            gbs = (w_bytes + kv) / (ms_tok / 1e3) / 1e9
            sweep.append({"weights": "q8_0" if key == "c2" else "f32", "ctx": ctx, "tok_s": 1e3 / ms_tok,
                          "ms_per_token": ms_tok, "bytes_per_token": w_bytes + kv, "kv_bytes": kv,
                          "hbm_gbs": gbs, "hbm_frac": gbs / peak,
                          "path": "decode kernel" if lib.jyc_model_decode_path(m.h) == 2 else "generic kernels"})
        m.close()
        del hw
    clk = clocks.stop()
    head = next(r for r in sweep if r["weights"] == "q8_0" and r["ctx"] == 4096)
    line = {
        "metric": "batch-1 decode tok/s (configs[2])", "value": head["tok_s"], "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_token"] * DECODE_C2,
        "higher_is_better": True, "scaling": "weak", "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"configs[2] Llama-3.2-1B shape, Q8_0 and fp32 weights (N(0, 0.02), seeded): "
                               f"batch-1 greedy decode of {DECODE_C2} tokens per step at seeded KV contexts "
                               f"1024 / 4096 / 16384; prefill of a 2048-token random prompt",
                   "l2": "inputs larger than L2 (1.3 GB / 4.9 GB of weights per token)"},
        "roofline": {"bound": "hbm", "kernel": head["path"], "achieved": head["hbm_gbs"], "peak": peak,
                     "unit": "GB/s", "frac": head["hbm_frac"], "bytes_per_launch": head["bytes_per_token"],
                     "launch_ms": head["ms_per_token"], "peak_kind": peak_kind, "traffic": None},
        "sweep": sweep, "prefill": prefill,
        "gpu_launches": int(lib.jyc_kernel_launches() - launches0), "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c3", choices=["c3", "c1", "c2", "c4", "prefill", "kquant"],
                    help="c3: the headline (configs[3] decode at context 4096, tensor parallel under "
                         "torchrun); c1: configs[1] decode; c2: configs[2] decode at contexts 1024 / 4096 / "
                         "16384 (Q8_0 and fp32) + its 2048-token prefill; c4: configs[4] batched decode sweep; "
                         "prefill: prompt prefill of --model; kquant: K-quant matmul bandwidth")
    ap.add_argument("--model", default="c1", choices=["c1", "c2", "c3"], help="prefill workload: which config")
    ap.add_argument("--seqs", default="1,4,16,32,64", help="c4: sequence counts of the sweep")
    ap.add_argument("--nvtx", action="store_true", help="mark the timed region as NVTX range 'timed' (profiling)")
    ap.add_argument("--decode-tokens", type=int, default=128, help="c4: greedy tokens per sequence per step")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload == "c3":
        return run_headline(args)
    if args.workload == "c4":
        return run_c4(args)
    if args.workload == "c2":
        return run_c2(args)
    if args.workload == "kquant":
        return run_kquant(args)
    if args.workload == "prefill":
        return run_prefill(args)
    return run_c1(args)


if __name__ == "__main__":
    sys.exit(main())
