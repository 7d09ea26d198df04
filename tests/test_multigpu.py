"""Tensor-parallel GPU tests: the fused NVLink collectives and a TP=2 model, run as one
process per GPU (tests/mp_fused_collectives.py under torch.distributed.run)."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(900)
@pytest.mark.parametrize("world", [1, 2, 4, 8])  # one rank still runs every kernel, pushing to itself
def test_fused_collectives_and_tp_model(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(ROOT, "tests", "mp_fused_collectives.py")]
    res = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]
    assert res.stdout.count(": ok") == world
