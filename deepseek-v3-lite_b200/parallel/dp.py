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

    def _broadcast_params(self) -> None:
        """Start every rank from rank 0's weights (and router biases)."""
        for f in self.engine.flats:
            dist.broadcast(f.master, src=0, group=self.group)
            f.refresh_shadow()
        for moe in self.engine.model.moe_layers():
            dist.broadcast(moe.gate.bias, src=0, group=self.group)

    def reduce_gradients(self) -> None:
        for f in self.engine.flats:
            dist.all_reduce(f.grad, op=dist.ReduceOp.AVG, group=self.group)

    def extra_sqsum(self) -> Optional[torch.Tensor]:
        return None

    def after_step(self) -> None:
        return None

    def global_counts(self, counts: torch.Tensor) -> torch.Tensor:
        c = counts.clone()
        dist.all_reduce(c, op=dist.ReduceOp.SUM, group=self.group)
        return c
