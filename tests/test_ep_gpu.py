"""Expert-parallel dispatch / combine kernels on B200.

* one rank: the peer-memory kernels store into the rank's own heap; the
  routed-expert layer (forward + backward, twice) is checked against fp32
  PyTorch;
* a wait on a flag no peer raises returns with the peer-timeout status after
  its short budget (the context stays usable);
* 2 ranks (when the box shows two GPUs): the same layer over real peer memory,
  and the training engine with experts spread vs replicated.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

PKG = Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200"


@pytest.mark.parametrize("balanced", [True, False], ids=["balanced", "owner"])
def test_ep_single_rank_layer_matches_fp32(balanced):
    from parallel.ep_selftest import run
    assert run(E=8, k=2, D=256, I=128, T=512, iters=2, verbose=False, balanced=balanced)


@pytest.mark.parametrize("balanced", [True, False], ids=["balanced", "owner"])
def test_ep_single_rank_uneven_experts(balanced):
    from parallel.ep_selftest import run
    assert run(E=5, k=3, D=128, I=128, T=300, iters=2, verbose=False, balanced=balanced)


def test_ep_wait_times_out_without_peer_signal():
    from ops._ext import native
    from parallel.ep import PH_COMBINE, ExpertParallel
    C = native()
    C.status_reset()
    ep = ExpertParallel(4, 2, 64, 128, n_slots=1, timeout_s=0.2)
    C.ep_wait(ep.heap.peers, ep.offs(0), ep.dims, PH_COMBINE, ep.expect)
    assert C.status_read() == 4          # DSV3_ERR_WAIT_PEER: the wait gave up, no hang
    C.status_reset()
    x = torch.ones(8, device="cuda")
    assert float((x * 2).sum()) == 16.0   # the context is still usable
    ep.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(args, n):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(PKG))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "parallel.ep_selftest"] + args
    return subprocess.run(cmd, cwd=PKG, env=env, capture_output=True, text=True, timeout=400)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_layer():
    r = _torchrun([], 2)
    assert r.returncode == 0 and "EP_SELFTEST OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_engine_matches_replicated_experts():
    r = _torchrun(["--engine"], 2)
    assert r.returncode == 0 and "EP_SELFTEST OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_sharded_experts_match_replicated():
    r = _torchrun(["--shard"], 2)
    assert r.returncode == 0 and "EP_SELFTEST OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
