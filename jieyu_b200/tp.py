"""Tensor-parallel decode across the GPUs of one node (configs[3] shape).

Sharding (one process per GPU, torch.distributed over NCCL for the plumbing):
rank r of t holds query heads [r H/t, (r+1) H/t) and kv heads
[r KV/t, (r+1) KV/t) (Q, K, V rows and biases), gate/up rows [r F/t, ..), and
the matching INPUT columns of O (q_dim/t) and down (F/t), so attention and the
int8 KV cache are rank-local; the LM head keeps rows [r V/t, (r+1) V/t) of
the vocabulary; norms and the embedding are whole on every rank. A rank's
shard is an ordinary smaller model for the C ABI; the cross-rank steps are
the sums of the O and down projections' partial outputs (two per layer) and
the largest of the ranks' argmaxes over their vocabulary slices.

A decode token is one launch of the decode kernel per rank: after its O and
down projections every CTA stores its partial rows into every rank's receive
area (peer stores over NVLink into CUDA-IPC-mapped memory) and counts itself
in that rank's arrival counter; the next phase waits (bounded) for all
ranks and adds their partials in rank order. (The "nccl" mode instead runs
half-layer windows of the kernel with NCCL all-reduces between them, in one
CUDA graph.) The residual stream stays identical on every rank (same sums in
the same order), so every rank emits the same token.

The reference (libs/model_libs/transformer_layer.h:10-90) runs the same math
on one host; the split is a column/row partition of its matrices.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import replace

import numpy as np

from . import _capi
from ._capi import check
from .model import Config, DeviceModel, HostWeights

Q8_BLOCK = 34


def _q8_rows(blob: np.ndarray, k: int, r0: int, r1: int) -> np.ndarray:
    """Rows [r0, r1) of a Q8_0 matrix [rows][k/32 blocks of 34 B]."""
    per = (k // 32) * Q8_BLOCK
    return np.ascontiguousarray(blob[r0 * per:r1 * per])


def _q8_cols(blob: np.ndarray, rows: int, k: int, c0: int, c1: int) -> np.ndarray:
    """Input columns [c0, c1) (multiples of 32) of a Q8_0 matrix, all rows."""
    m = blob.reshape(rows, k // 32, Q8_BLOCK)
    return np.ascontiguousarray(m[:, c0 // 32:c1 // 32, :]).reshape(-1)


def shard_config(cfg: Config, size: int) -> Config:
    if cfg.heads % size or cfg.kv_heads % size:
        raise ValueError(f"{cfg.name}: heads {cfg.heads} / kv heads {cfg.kv_heads} not divisible by {size}")
    if (cfg.heads // size * cfg.head_dim) % 32 or (cfg.inter // size) % 32:
        raise ValueError(f"{cfg.name}: per-rank O / down input columns must be whole Q8_0 blocks")
    return replace(cfg, heads=cfg.heads // size, kv_heads=cfg.kv_heads // size, inter=cfg.inter // size,
                   name=f"{cfg.name}_tp{size}")


def shard_weights(hw: HostWeights, rank: int, size: int, shard_head: bool = True) -> HostWeights:
    """Rank `rank`'s shard of Q8_0 host weights (see the module docstring);
    shard_head=False keeps the whole LM head (the "nccl" mode, whose head
    window picks the token from the rank's own logits)."""
    cfg = hw.cfg
    if cfg.wtype != "q8":
        raise ValueError("tensor parallelism is built for Q8_0 weights")
    sc = shard_config(cfg, size)
    D, hd = cfg.hidden, cfg.head_dim
    q0, q1 = rank * sc.q_dim, (rank + 1) * sc.q_dim
    k0, k1 = rank * sc.kv_dim, (rank + 1) * sc.kv_dim
    f0, f1 = rank * sc.inter, (rank + 1) * sc.inter
    t = {}
    for l in range(cfg.layers):
        t[f"rms1.{l}"] = hw.t[f"rms1.{l}"]
        t[f"rms2.{l}"] = hw.t[f"rms2.{l}"]
        t[f"q.{l}"] = _q8_rows(hw.t[f"q.{l}"], D, q0, q1)
        t[f"k.{l}"] = _q8_rows(hw.t[f"k.{l}"], D, k0, k1)
        t[f"v.{l}"] = _q8_rows(hw.t[f"v.{l}"], D, k0, k1)
        t[f"o.{l}"] = _q8_cols(hw.t[f"o.{l}"], D, cfg.q_dim, q0, q1)
        t[f"gate.{l}"] = _q8_rows(hw.t[f"gate.{l}"], D, f0, f1)
        t[f"up.{l}"] = _q8_rows(hw.t[f"up.{l}"], D, f0, f1)
        t[f"down.{l}"] = _q8_cols(hw.t[f"down.{l}"], D, cfg.inter, f0, f1)
        if cfg.qkv_bias:
            t[f"bq.{l}"] = np.ascontiguousarray(hw.t[f"bq.{l}"][q0:q1])
            t[f"bk.{l}"] = np.ascontiguousarray(hw.t[f"bk.{l}"][k0:k1])
            t[f"bv.{l}"] = np.ascontiguousarray(hw.t[f"bv.{l}"][k0:k1])
    # LM head: rank r keeps vocabulary rows [r V/t, (r+1) V/t); the embedding
    # stays whole (a tied embedding becomes a separate whole Q8_0 copy)
    V = cfg.vocab
    if shard_head and V % size == 0 and (V // size) % 16 == 0:
        v0, v1 = rank * V // size, (rank + 1) * V // size
        t["head"] = _q8_rows(hw.t["head"], D, v0, v1)
        t["embed"] = hw.t["head"] if cfg.embed == "tied" else hw.t["embed"]
        sc = replace(sc, vocab=v1 - v0, embed_rows=V, vocab_offset=v0,
                     embed="q8" if cfg.embed == "tied" else cfg.embed)
    else:
        t["head"] = hw.t["head"]
        if "embed" in hw.t:
            t["embed"] = hw.t["embed"]
    t["final_norm"] = hw.t["final_norm"]
    return HostWeights(sc, t, hw.cos, hw.sin)


class _DevBuf:
    """A device buffer of the library seen by torch (zero copy)."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


class TPDecoder:
    """One rank of a tensor-parallel decode (call collectively on every rank).

    mode "kernel" (default): one decode-kernel launch per token; the kernel
    exchanges the O and down partials with the other ranks itself (peer
    stores over NVLink into CUDA-IPC-mapped receive areas, bounded waits).
    mode "nccl": half-layer windows of the decode kernel with NCCL
    all-reduces of the partials between them, captured in a CUDA graph."""

    def __init__(self, hw_full: HostWeights, rank: int, size: int, group=None, mode: str = "kernel"):
        import torch
        import torch.distributed as dist

        self.torch, self.dist, self.group = torch, dist, group
        self.rank, self.size, self.mode = rank, size, mode
        self.cfg = hw_full.cfg
        self.shard = shard_weights(hw_full, rank, size, shard_head=(mode == "kernel"))
        self.m = DeviceModel(self.shard)
        self.lib = _capi.load()
        if self.lib.jyc_model_decode_path(self.m.h) != 2:
            raise RuntimeError("tensor-parallel decode needs the decode kernel (Q8_0 tiled layout)")
        self.stream = torch.cuda.Stream()
        self.graph = None
        if mode == "kernel":
            handle = (C.c_ubyte * 64)()
            check(self.lib.jyc_model_tp_open(self.m.h, size, rank, handle))
            handles = [None] * size
            dist.all_gather_object(handles, bytes(handle), group=group)
            allh = (C.c_ubyte * (64 * size)).from_buffer_copy(b"".join(handles))
            check(self.lib.jyc_model_tp_connect(self.m.h, allh))
            dist.barrier(group=group)
            return
        po, npo, pd, npd = C.c_void_p(), C.c_int(), C.c_void_p(), C.c_int()
        check(self.lib.jyc_model_partials(self.m.h, C.byref(po), C.byref(npo), C.byref(pd), C.byref(npd)))
        self.po = torch.as_tensor(_DevBuf(po.value, npo.value), device="cuda")
        self.pd = torch.as_tensor(_DevBuf(pd.value, npd.value), device="cuda")

    def _window(self, first: int, last: int) -> None:
        check(self.lib.jyc_model_decode_window(self.m.h, first, last, self.stream.cuda_stream))

    def _step(self) -> None:
        L = self.cfg.layers
        for l in range(L):
            self._window(2 * l, 2 * l + 1)
            self.dist.all_reduce(self.po, group=self.group)
            self._window(2 * l + 1, 2 * l + 2)
            self.dist.all_reduce(self.pd, group=self.group)
        self._window(2 * L, 2 * L + 1)

    def capture(self) -> bool:
        """nccl mode: records one token step (kernels + all-reduces) into a
        CUDA graph; False (and eager steps) if the capture is refused or in
        kernel mode (one launch per token needs no graph)."""
        torch = self.torch
        if self.mode == "kernel":
            return False
        with torch.cuda.stream(self.stream):
            self._step()  # warm-up outside capture (NCCL communicator setup)
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g, stream=self.stream):
                self._step()
        except RuntimeError:
            self.graph = None
            return False
        self.graph = g
        return True

    def step(self, n: int = 1) -> None:
        """n decode tokens on self.stream."""
        torch = self.torch
        if self.mode == "kernel":
            check(self.lib.jyc_decode_device(self.m.h, n, self.stream.cuda_stream))
            return
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                if self.graph is not None:
                    self.graph.replay()
                else:
                    self._step()

    def prefill_by_steps(self, prompt: np.ndarray) -> None:
        """Fills the KV cache with the prompt through decode steps (teacher
        forcing: the prompt ids are written into the device token buffer)."""
        torch = self.torch
        ids = torch.from_numpy(np.ascontiguousarray(prompt, dtype=np.int32)).cuda()
        tok_ptr = self.lib.jyc_model_tokens_device(self.m.h)
        toks = torch.as_tensor(_DevBuf(tok_ptr, self.cfg.max_seq + 1, "<i4"), device="cuda")
        with torch.cuda.stream(self.stream):
            for i in range(len(prompt)):
                toks[: i + 1].copy_(ids[: i + 1])
                check(self.lib.jyc_model_rewind(self.m.h, i + 1, self.stream.cuda_stream))
                self.step(1)
        self.stream.synchronize()

    def prefill(self, prompt: np.ndarray) -> None:
        """Tensor-parallel prefill (call on every rank): the prompt's first
        T - 1 tokens run in passes of the batched prefill, each pass as
        half-layer windows with an NCCL all-reduce (sum) of the shards' O and
        down partial rows between them; the last layer's MLP half is skipped
        (no KV entry depends on it). The last prompt token then goes through
        one tensor-parallel decode step, which writes its KV entries and
        appends the first new token (the LM head's argmax over the ranks'
        vocabulary slices)."""
        torch, dist = self.torch, self.dist
        T = len(prompt)
        ids = torch.from_numpy(np.ascontiguousarray(prompt, dtype=np.int32)).cuda()
        tok_ptr = self.lib.jyc_model_tokens_device(self.m.h)
        toks = torch.as_tensor(_DevBuf(tok_ptr, self.cfg.max_seq + 1, "<i4"), device="cuda")
        part, cap = C.c_void_p(), C.c_int()
        check(self.lib.jyc_model_prefill_partial(self.m.h, C.byref(part), C.byref(cap)))
        D, L = self.cfg.hidden, self.cfg.layers
        pbuf = torch.as_tensor(_DevBuf(part.value, cap.value * D), device="cuda")
        s = self.stream.cuda_stream
        with torch.cuda.stream(self.stream):
            toks[:T].copy_(ids)
            n = T - 1
            for start in range(0, n, cap.value):
                rows = min(cap.value, n - start)
                for p in range(2 * L - 1):
                    check(self.lib.jyc_model_prefill_window(self.m.h, start, rows, p, p + 1, s))
                    if p + 1 < 2 * L - 1:
                        dist.all_reduce(pbuf[: rows * D], group=self.group)
            check(self.lib.jyc_model_rewind(self.m.h, T, s))
            self.step(1)

    def generate(self, prompt: np.ndarray, max_new: int, cb=None) -> np.ndarray:
        """The tensor-parallel counterpart of generate() (generate.h:90-112,
        greedy; call on every rank): the prompt ids go from pinned host
        memory to the device, the tensor-parallel prefill appends the first
        new id, then decode steps run in blocks of 1, 2, 4, .. 32 tokens,
        each block's ids read back to the host and handed to cb in order
        (every rank runs the same blocks and holds the same ids). Stops after
        max_new ids or at the context limit; returns prompt + new ids."""
        torch = self.torch
        T = len(prompt)
        pin = torch.from_numpy(np.ascontiguousarray(prompt, dtype=np.int32)).pin_memory()
        max_new = min(max_new, self.cfg.max_seq - T)
        out = list(np.asarray(prompt, dtype=np.int32))
        if max_new <= 0:
            return np.asarray(out, dtype=np.int32)
        self.prefill(pin.numpy())
        tok_ptr = self.lib.jyc_model_tokens_device(self.m.h)
        toks = torch.as_tensor(_DevBuf(tok_ptr, self.cfg.max_seq + 1, "<i4"), device="cuda")
        host = torch.empty(self.cfg.max_seq + 1, dtype=torch.int32).pin_memory()
        done, have, block = 1, T, 1
        while True:
            n_new = T + done - have
            with torch.cuda.stream(self.stream):
                host[have:have + n_new].copy_(toks[have:have + n_new], non_blocking=True)
            self.stream.synchronize()
            for i in range(have, have + n_new):
                out.append(int(host[i]))
                if cb is not None:
                    cb(int(host[i]))
            have += n_new
            if done >= max_new:
                break
            n = min(block, max_new - done)
            self.step(n)
            done += n
            block = min(2 * block, 32)
        return np.asarray(out, dtype=np.int32)

    def tokens(self, n: int) -> np.ndarray:
        torch = self.torch
        self.stream.synchronize()
        tok_ptr = self.lib.jyc_model_tokens_device(self.m.h)
        toks = torch.as_tensor(_DevBuf(tok_ptr, self.cfg.max_seq + 1, "<i4"), device="cuda")
        return toks[:n].cpu().numpy()

    def close(self) -> None:
        self.graph = None
        self.m.close()
