"""Peer-memory data-parallel optimizer step (reduce-scatter + sharded AdamW +
all-gather, csrc/dp.cu) vs the NCCL all-reduce step, on two GPUs."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

PKG = Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_dp_step_matches_nccl_all_reduce():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(PKG))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "parallel.dp_selftest"]
    r = subprocess.run(cmd, cwd=PKG, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0 and "DP_SELFTEST OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
