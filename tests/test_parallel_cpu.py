"""Data-parallel control plane on CPU ranks (gloo, world size 2).

The fused engine itself needs a B200; what is tested here is the host-side
logic every rank runs: weight broadcast from rank 0, gradient averaging,
global expert counts for the router-bias update, and failure detection when a
peer disappears (the survivor's next collective errors out within the group
timeout instead of hanging).
"""
import datetime
import os
import socket
import sys
import traceback
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SRC = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "deepseek-v3-lite_b200")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    sys.path.insert(0, SRC)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


class _Flat:
    def __init__(self, n, rank):
        self.master = torch.full((n,), float(rank + 1))
        self.grad = torch.arange(n, dtype=torch.float32) * (rank + 1)
        self.refreshed = 0

    def refresh_shadow(self):
        self.refreshed += 1


class _Moe:
    def __init__(self, rank):
        self.gate = SimpleNamespace(bias=torch.full((4,), 0.5 * rank))


def _dp_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from parallel.dp import DataParallel
        flats = [_Flat(8, rank), _Flat(3, rank)]
        model = SimpleNamespace(moe_layers=lambda: [_Moe(rank)])
        eng = SimpleNamespace(flats=flats, model=model)
        moes = model.moe_layers()
        eng.model = SimpleNamespace(moe_layers=lambda: moes)
        dp = DataParallel(eng)
        assert dp.world_size == world and dp.rank == rank
        assert torch.equal(flats[0].master, torch.full((8,), 1.0))          # rank 0's weights everywhere
        assert torch.equal(moes[0].gate.bias, torch.zeros(4))               # and router bias
        assert flats[0].refreshed == 1
        dp.reduce_gradients()
        mean = sum(r + 1 for r in range(world)) / world
        assert torch.allclose(flats[0].grad, torch.arange(8, dtype=torch.float32) * mean)
        counts = torch.tensor([rank, 1, 2, 3], dtype=torch.int32)
        assert torch.equal(dp.global_counts(counts), torch.tensor([sum(range(world)), world, 2 * world, 3 * world],
                                                                  dtype=torch.int32))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(fn, world=2, extra=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + tuple(extra)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    return out


def test_data_parallel_control_plane():
    out = _run(_dp_worker)
    assert out == {0: "ok", 1: "ok"}, out


def _dead_peer_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        dist.barrier()
        if rank == 1:
            # leaves between steps: nothing in flight, never joins the next collective
            q.put((rank, "left"))
            q.close()
            q.join_thread()          # flush the message before the hard exit
            os._exit(0)
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            q.put((rank, "no error"))
        except Exception as exc:  # the survivor learns of the loss on the host
            q.put((rank, f"detected: {type(exc).__name__}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_dead_peer_is_detected_not_hung():
    out = _run(_dead_peer_worker)
    assert out[1] == "left"
    assert out[0].startswith("detected"), out[0]
