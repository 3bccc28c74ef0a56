"""Tensor-parallel decode worker (run under torchrun, one rank per GPU).

A configs[3]-shaped model (32 query heads, 8 kv heads, head_dim 128, FFN
14336) with 2 layers and a 4096-token vocabulary: every rank decodes through
its shard (jieyu_b200.tp.TPDecoder, NCCL all-reduces between decode-kernel
windows); rank 0 then decodes the same prompt with the whole model on one GPU
and compares the greedy sequences. Prints TP_OK on success.
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


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    cfg = replace(CONFIGS["c3"], layers=2, vocab=4096, max_seq=256, name="c3_2layer")
    hw = HostWeights.synthetic(cfg)
    prompt = prompt_ids(cfg, n=8)
    new = 16
    mode = os.environ.get("JIEYU_TP_MODE", "kernel")
    tp = TPDecoder(hw, rank, world, mode=mode)
    graphed = tp.capture()
    tp.prefill_by_steps(prompt)      # KV of the prompt + the first new token
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
        res["tp"] = [int(x) for x in got]
        res["one_gpu"] = [int(x) for x in ref]
        ok = list(ref) == list(got)
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
