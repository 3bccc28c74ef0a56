"""Tensor-parallel decode worker (run under torchrun, one rank per GPU).

A configs[3]-shaped model (32 query heads, 8 kv heads, head_dim 128, FFN
14336) with 2 layers and a 4096-token vocabulary: every rank decodes through
its shard (jieyu_b200.tp.TPDecoder: the in-kernel exchange, or NCCL
all-reduces between decode-kernel windows; JIEYU_TP_MODE=prefill runs a
700-token prompt through the tensor-parallel batched prefill first); rank 0
replays the sharded sequence through the whole model on one GPU (each new
token must be its argmax on that history, or a near tie: at most 2 of 16) and
reports the single-GPU sequence beside it. Prints TP_OK on success.
"""
import datetime
import json
import os
import sys
import time
from dataclasses import replace

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from jieyu_b200.model import CONFIGS, DeviceModel, HostWeights, prompt_ids  # noqa: E402
from jieyu_b200.tp import TPDecoder  # noqa: E402


def replay(hw, seq, prompt_len):
    """Every token the sharded model appended, replayed on that sequence's
    own history through the whole model on one GPU (teacher forced; its
    logits are pinned to the reference by tests/test_gpu_model.py): (tokens
    that are neither its argmax nor a near tie, near ties). A near tie is a
    top-2 gap below twice LOGIT_TOL of max|logit|, the model tests' bar: the
    shards' partial sums change the fp32 summation order, which may flip
    such a pick."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from _util import LOGIT_TOL
    m = DeviceModel(hw)
    bad, ties = [], 0
    try:
        tok = np.ascontiguousarray(seq[:prompt_len], np.int32)
        pos = 0
        for i in range(prompt_len, len(seq)):
            want = m.forward_logits(tok, pos)
            pos += len(tok)
            best = int(np.argmax(want))
            if int(seq[i]) != best:
                top2 = np.sort(want)[-2:]
                if top2[1] - top2[0] < 2 * LOGIT_TOL * np.abs(want).max():
                    ties += 1
                else:
                    bad.append((i, int(seq[i]), best))
            tok = np.array([seq[i]], np.int32)
    finally:
        m.close()
    return bad, ties


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    mode = os.environ.get("JIEYU_TP_MODE", "kernel")
    prefill = mode == "prefill"  # tensor-parallel batched prefill (kernel-mode decode after it)
    # prefill: a prompt longer than one batched pass (512 tokens), 2 passes
    cfg = replace(CONFIGS["c3"], layers=2, vocab=4096, max_seq=1100 if prefill else 256, name="c3_2layer")
    hw = HostWeights.synthetic(cfg)
    prompt = prompt_ids(cfg, n=700 if prefill else 8)
    new = 16
    tp = TPDecoder(hw, rank, world, mode="kernel" if prefill else mode)
    graphed = tp.capture()
    if prefill:
        tp.prefill(prompt)           # KV of the prompt + the first new token
    else:
        tp.prefill_by_steps(prompt)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    tp.step(new - 1)
    tp.stream.synchronize()
    dt = time.perf_counter() - t0
    got = tp.tokens(len(prompt) + new)
    tp.close()
    dist.barrier()
    ok = True
    res = {"world": world, "mode": mode, "graphed": graphed, "tp_ms_per_token": dt * 1e3 / (new - 1)}
    if rank == 0:
        ref = DeviceModel(hw).generate(prompt, new)
        res["tp"] = [int(x) for x in got[len(prompt):]]
        res["one_gpu"] = [int(x) for x in ref[len(prompt):]]
        bad, ties = replay(hw, got, len(prompt))
        res["mismatches"], res["near_ties"] = bad, ties
        ok = not bad and ties <= 2
        res["match"] = ok
        print(json.dumps(res), flush=True)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0 and flag.item() == 1:
        print("TP_OK", flush=True)
    return 0 if flag.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
