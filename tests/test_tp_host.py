"""Host side of tensor parallelism on CPU: the weight shards re-assemble the
model, and the row-split partial sums all-reduced over 2 gloo ranks equal the
whole product (the math the decode's O / down all-reduces rely on)."""
import os
import socket

import numpy as np
import pytest

from jieyu_b200.model import Config, HostWeights, synth_f32
from jieyu_b200.tp import shard_config, shard_weights

CFG = Config("tp_small", 256, 2, 8, 4, 64, 512, 1024, 1e4, "q8", "f32", False, 64, 4, 4)


def _blocks(blob, rows, k):
    return blob.reshape(rows, k // 32, 34)


@pytest.mark.parametrize("size", [2, 4])
def test_shards_reassemble_the_model(size):
    hw = HostWeights.synthetic(CFG)
    shards = [shard_weights(hw, r, size) for r in range(size)]
    D, q, kv, F = CFG.hidden, CFG.q_dim, CFG.kv_dim, CFG.inter
    for l in range(CFG.layers):
        for name, rows in (("q", q), ("k", kv), ("v", kv), ("gate", F), ("up", F)):
            whole = np.concatenate([s.t[f"{name}.{l}"] for s in shards])
            assert np.array_equal(whole, hw.t[f"{name}.{l}"]), name
        for name, k in (("o", q), ("down", F)):
            whole = np.concatenate([_blocks(s.t[f"{name}.{l}"], D, k // size) for s in shards], axis=1)
            assert np.array_equal(whole, _blocks(hw.t[f"{name}.{l}"], D, k)), name
    sc = shards[0].cfg
    assert (sc.heads, sc.kv_heads, sc.inter) == (CFG.heads // size, CFG.kv_heads // size, CFG.inter // size)
    # vocabulary-sharded LM head: the slices re-assemble it, the embedding stays whole
    if CFG.vocab % size == 0 and (CFG.vocab // size) % 16 == 0:
        assert np.array_equal(np.concatenate([s.t["head"] for s in shards]), hw.t["head"])
        assert [s.cfg.vocab_offset for s in shards] == [r * CFG.vocab // size for r in range(size)]
        assert all(s.cfg.embed_rows == CFG.vocab for s in shards)
    else:
        assert shards[0].t["head"] is hw.t["head"]


def test_shard_config_rejects_uneven_splits():
    with pytest.raises(ValueError):
        shard_config(CFG, 3)
    with pytest.raises(ValueError):
        shard_config(Config("odd_ffn", 256, 1, 8, 4, 64, 1376, 1000, 1e4), 2)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    D, K = 64, 256
    w = synth_f32(7, 1, D * K, 1.0).reshape(D, K)
    x = synth_f32(7, 2, K, 1.0)
    c0, c1 = rank * K // world, (rank + 1) * K // world
    part = torch.from_numpy(w[:, c0:c1] @ x[c0:c1]).contiguous()   # rank's input columns
    dist.all_reduce(part)
    q.put((rank, part.numpy()))
    dist.destroy_process_group()


def test_row_split_partials_allreduce_on_gloo():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    D, K = 64, 256
    w = synth_f32(7, 1, D * K, 1.0).reshape(D, K)
    x = synth_f32(7, 2, K, 1.0)
    want = w @ x
    for r in range(2):
        assert np.allclose(out[r], want, rtol=1e-5, atol=1e-4)
    assert np.array_equal(out[0], out[1])  # every rank holds the same sum
