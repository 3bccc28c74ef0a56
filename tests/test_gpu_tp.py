"""Tensor-parallel decode on 2 GPUs (skipped with fewer): every greedy token
of the sharded decode is the whole model's argmax on the same history, or a
near tie (tests/tp_worker.py),
with the in-kernel NVLink exchange, with NCCL between kernel windows, and
after a tensor-parallel batched prefill (NCCL all-reduce of the shards' O and
down partial rows, two prefill passes)."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["kernel", "nccl", "prefill"])
def test_tp2_decode_matches_single_gpu(cuda, mode):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", JIEYU_TP_MODE=mode)
    if mode == "prefill":
        env["JYC_PF_ROWS"] = "512"  # the 700-token prompt in two passes
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "TP_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
