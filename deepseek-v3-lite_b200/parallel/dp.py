"""Data parallelism for the fused training engine.

Every rank holds the full parameter set in the engine's flat buffers.  At the
accumulation boundary the fp32 gradient buffers are averaged over the group
(one NCCL all-reduce per flat buffer, i.e. two large bucketed collectives per
step); the global gradient norm is then the local one, every rank runs the
same fused AdamW and stays bit-identical.  The aux-loss-free router bias is
updated from the *global* expert counts (all-reduced), so routing stays
identical on every rank.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch
import torch.distributed as dist


class DataParallel:
    def __init__(self, engine, group=None):
        self.engine = engine
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._broadcast_params()

    def _replicated(self):
        return [f for f in self.engine.flats if not getattr(f, "rank_local", False)]

    def _rank_local(self):
        return [f for f in self.engine.flats if getattr(f, "rank_local", False)]

    def _broadcast_params(self) -> None:
        """Start every rank from rank 0's weights (and router biases); a rank's
        own routed experts (when sharded) are its own."""
        for f in self._replicated():
            dist.broadcast(f.master, src=0, group=self.group)
            f.refresh_shadow()
        for moe in self.engine.model.moe_layers():
            dist.broadcast(moe.gate.bias, src=0, group=self.group)

    def reduce_gradients(self) -> None:
        for f in self._replicated():
            dist.all_reduce(f.grad, op=dist.ReduceOp.AVG, group=self.group)
        # a sharded expert's gradient is complete on its owner (every rank's
        # tokens reached it); the data-parallel mean divides it by the ranks
        for f in self._rank_local():
            f.grad.mul_(1.0 / self.world_size)

    def extra_sqsum(self) -> Optional[torch.Tensor]:
        """Squared gradient norm of the other ranks' sharded experts."""
        local = self._rank_local()
        if not local:
            return None
        from ops._ext import native
        t = torch.zeros(1, device=local[0].grad.device)
        native().grad_sqsum([f.grad for f in local], torch.empty(1024 * len(local), device=t.device), t)
        tot = t.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM, group=self.group)
        return tot - t

    def after_step(self) -> None:
        return None

    def global_counts(self, counts: torch.Tensor) -> torch.Tensor:
        c = counts.clone()
        dist.all_reduce(c, op=dist.ReduceOp.SUM, group=self.group)
        return c


def _shard(n: int, rank: int, world: int, align: int = 64) -> tuple:
    """Contiguous, 64-element aligned shard [lo, hi) of n elements owned by rank."""
    def cut(r):
        return min(n, (r * n // world + align - 1) // align * align)
    return cut(rank), cut(rank + 1)


class FusedDataParallel(DataParallel):
    """Data parallelism whose optimizer step runs over NVLink peer memory.

    The flat fp32 gradient / fp32 master / bf16 shadow buffers of every rank
    sit in one symmetric heap.  ``step`` replaces all-reduce + full AdamW with
    (csrc/dp.cu): a barrier (every rank's gradients complete), a
    reduce-scatter that averages this rank's shard straight from the peers'
    buffers and takes its squared norm, an exchange of the norms (same clip
    coefficient everywhere), and AdamW on the shard only, whose new master and
    bf16 shadow values are stored into every rank's buffers (the
    all-gather), then a closing barrier.  Each rank allocates and advances
    the Adam moments of its own shard only (ZeRO-1: 8 bytes per replicated
    parameter per rank become 8 / ranks); ``gather_moments`` assembles the
    full moments for the duration of a checkpoint write.
    """

    PH_READY, PH_NORM, PH_GATHERED = 0, 1, 2

    @staticmethod
    def make_heap(numels):
        """Symmetric heap holding the flat buffers of the given sizes plus the
        step's flags; returns (heap, alloc_0, alloc_1, ...)."""
        from .symm import SymmetricHeap, heap_layout
        sizes = [4 * 8 * 4, 8 * 4]                      # flags [4 phases][8 ranks], norm partials [8]
        for n in numels:
            sizes += [n * 4, n * 4, n * 2]              # master, grad, shadow
        offs = heap_layout(sizes)
        heap = SymmetricHeap(offs[-1])
        heap.dp_offs = offs
        allocs = []
        for i, n in enumerate(numels):
            base = 2 + 3 * i
            table = {"master": (offs[base], torch.float32), "grad": (offs[base + 1], torch.float32),
                     "shadow": (offs[base + 2], torch.bfloat16)}

            def alloc(name, numel, dtype, table=table, n=n):
                off, dt = table[name]
                assert numel == n and dtype == dt
                return heap.tensor(off, (numel,), dtype)
            allocs.append(alloc)
        return (heap, *allocs)

    def __init__(self, engine, heap, group=None):
        import os
        from ops._ext import native
        self.heap = heap
        self.C = native()
        self.offs = [heap.dp_offs[0], heap.dp_offs[1]]
        self.budget_ns = int(float(os.environ.get("DSV3_DP_TIMEOUT_S", "60")) * 1e9)
        super().__init__(engine, group=group)
        self.n_heap = len(self._replicated())   # the heap holds the replicated flats, first in engine.flats
        self.shards = [_shard(f.numel, self.rank, self.world_size) for f in engine.flats[:self.n_heap]]
        self.flat_offs = [(heap.dp_offs[2 + 3 * i], heap.dp_offs[3 + 3 * i], heap.dp_offs[4 + 3 * i])
                          for i in range(self.n_heap)]
        dev = engine.flats[0].master.device
        self.expect = torch.zeros(4 * 8, dtype=torch.int32, device=dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        opt = engine.optimizer
        for fi, (lo, hi) in enumerate(self.shards):
            opt.shard_moments(fi, lo, hi)
        # optimizer.step() runs this rank's part of the data-parallel step
        self.max_norm = float(getattr(engine.config, "max_grad_norm", 1.0))
        opt.stepper = lambda o: self.step(o, self.max_norm)

    def _args(self):
        return self.heap.peers, self.offs, self.rank, self.budget_ns

    def reduce_gradients(self) -> None:
        """Plain all-reduce of the full gradients (diagnostics and tests; the
        training step uses ``step``)."""
        super().reduce_gradients()

    def step(self, optimizer, max_norm: float) -> None:
        C = self.C
        peers, offs, me, budget = self._args()
        C.dp_barrier(peers, offs, me, budget, self.PH_READY, self.expect)
        self.sq.zero_()
        for (lo, hi), (_, off_g, _) in zip(self.shards, self.flat_offs):
            C.dp_reduce(peers, offs, me, budget, off_g, lo, hi, 1.0 / self.world_size, self.sq)
        local = self._rank_local()
        if local:
            # sharded experts: the owner's gradient / ranks, its norm joins the exchange
            for f in local:
                f.grad.mul_(1.0 / self.world_size)
            t = torch.zeros(1, device=self.sq.device)
            C.grad_sqsum([f.grad for f in local], torch.empty(1024 * len(local), device=t.device), t)
            self.sq.add_(t)
        C.dp_norm(peers, offs, me, budget, self.sq, self.expect, float(max_norm), optimizer.grad_norm, optimizer.clip)
        optimizer.step_count += 1
        for fi in range(self.n_heap):
            f = optimizer.flats[fi]
            group = optimizer.param_groups[optimizer.flat_groups[fi]]
            lo, hi = self.shards[fi]
            off_m, off_g, off_s = self.flat_offs[fi]
            b1, b2 = group["betas"]
            n_decay = f.numel if group["weight_decay"] > 0 else 0
            C.dp_update(peers, offs, me, budget, off_m, off_g, off_s, optimizer.exp_avg[fi], optimizer.exp_avg_sq[fi],
                        lo, hi, n_decay, float(group["lr"]), float(b1), float(b2), float(group["eps"]),
                        float(group["weight_decay"]), optimizer.step_count, optimizer.clip)
        for fi in range(self.n_heap, len(optimizer.flats)):
            optimizer.step_flat(fi)            # this rank's experts: plain local AdamW
        optimizer.mark_step()
        C.dp_barrier(peers, offs, me, budget, self.PH_GATHERED, self.expect)

    def gather_moments(self, optimizer) -> dict:
        """Every rank's moment shards -> ``{flat index: (exp_avg, exp_avg_sq)}``
        full-size buffers on every rank (collective; the caller drops them)."""
        full = {}
        for fi, f in enumerate(optimizer.flats[:self.n_heap]):
            bufs = []
            for shard in (optimizer.exp_avg[fi], optimizer.exp_avg_sq[fi]):
                buf = torch.empty(f.numel, dtype=shard.dtype, device=shard.device)
                for r in range(self.world_size):
                    lo, hi = _shard(f.numel, r, self.world_size)
                    if hi > lo:
                        if r == self.rank:
                            buf[lo:hi].copy_(shard)
                        dist.broadcast(buf[lo:hi], src=r, group=self.group)
                bufs.append(buf)
            full[fi] = tuple(bufs)
        return full
