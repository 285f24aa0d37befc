"""The N-sharded gate/up (tensor-parallel MLP over NCCL) on 2 GPUs: the
forward is bit-identical to the single-GPU forward, eager and replayed from
a CUDA graph (worker: tests/_sharded_forward_worker.py).  Skipped on a host
with one GPU; the exchange logic itself is covered on CPU by
tests/test_multirank.py (gloo)."""

from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_forward_is_bit_identical_on_2_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "_sharded_forward_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "sharded ok" in res.stdout, res.stdout[-3000:]
