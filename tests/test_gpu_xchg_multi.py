"""Exchange across real GPUs (CUDA IPC peer mappings, stores over NVLink from the attention kernel):
runs tests/xchg_worker.py with one process per GPU on 2 GPUs; the `multicast`
case stores through an NVLink multicast address of symmetric memory.  Skipped on a
machine with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["heads", "balanced", "multicast"])
def test_exchange_two_gpus_matches_single_context(mode):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "xchg_worker.py"), mode]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    if "multicast unsupported" in p.stdout:
        pytest.skip("the GPUs offer no NVLink multicast object")
    assert "match" in p.stdout
