"""Expert parallelism for DeepSeekMoE over the GPUs of one NVSwitch box.

Routed experts are split into contiguous ranges, rank ``d`` of ``R`` owning
``[d*E//R, (d+1)*E//R)`` (uneven when ``R`` does not divide ``E``).  Where
the rows go depends on the layout:

* ``balanced`` (the default while expert weights are replicated): all ranks'
  rows in expert order, each expert's range padded to 256 rows, form one
  sequence that is cut into ``R`` equal contiguous shares; rank ``d``
  computes share ``d``.  Every rank runs the same number of expert rows
  whatever the routing (at random init some experts get several times the
  mean), an expert's rows may be split over two ranks, and each rank adds its
  rows' part of every touched expert's weight gradient;
* ``owner`` (sharded expert weights): rank ``d`` receives every row routed to
  the experts it owns and computes their weight gradients.

A MoE layer on every rank then runs

forward
  router GEMM + top-k (local) -> ``ep_plan``: all-gather of the per-expert
  counts over peer memory and the receive layout -> ``ep_dispatch``: each
  (token, slot) row stored straight into its expert owner's receive slot ->
  wait -> grouped SwiGLU GEMM and grouped down GEMM on the received rows
  (operands in local memory, tcgen05) whose epilogue also stores each output
  row into its home rank's combine inbox at the token's slot (the combine
  fused with the down projection; ``ep_send_back`` is the unfused variant) ->
  wait -> weighted combine into the fp32 residual (home side).
backward
  ``ep_dispatch_bwd``: the output-gradient rows take the forward routes ->
  wait -> ``ep_bwd_prep`` (dy = w * dout, dw = <dout, y>) -> grouped
  data/weight gradients -> ``ep_send_back`` of the input-gradient rows and
  the gate-weight gradients -> wait -> sum into the token gradients and the
  router backward (home side).

Every transfer is a plain store from a kernel into another GPU's memory
(no NCCL, no staging copy); every wait is bounded and reports through the
device status word.  Expert weights stay replicated; a rank computes weight
gradients only for the experts it owns (the others stay zero), so the data-
parallel gradient average yields exactly the global average and every rank
keeps identical weights and optimizer state (checkpoints need no gather).

No counterpart in the reference: its experts all live on one device
(models/moe.py:52-201).
"""
from __future__ import annotations

import math
import os
from typing import List, Optional, Sequence

import torch

from ops._ext import native

PH_COUNTS, PH_DISPATCH, PH_COMBINE, PH_BWD_DISPATCH, PH_BWD_COMBINE = range(5)
MAX_RANKS = 8
_FLAG_BYTES = 5 * MAX_RANKS * 4


def _pad(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def expert_range(rank: int, n_experts: int, world: int) -> tuple:
    """Routed experts owned by ``rank``: ``[lo, hi)``."""
    return rank * n_experts // world, (rank + 1) * n_experts // world


def owner_of(expert: int, n_experts: int, world: int) -> int:
    d = world - 1
    while d > 0 and d * n_experts // world > expert:
        d -= 1
    return d


def balanced_capacity(tokens: int, topk: int, n_experts: int, world: int) -> int:
    """Rows of one rank's receive slot in the balanced layout: its share of
    the largest possible padded sequence (every rank's ``tokens * topk`` rows
    plus up to 255 padding rows per expert), rounded up to 256."""
    total = world * tokens * topk + n_experts * 255
    return max(256, _pad(-(-total // world), 256))


def plan_reference_balanced(cnt_all: torch.Tensor, rank: int):
    """What ``ep_plan`` computes in the balanced layout, in plain PyTorch (CPU oracle).

    Returns ``(send_base [E] (global positions), row_off [E+1], recv_cnt [E],
    chunk, used)`` for ``rank``."""
    R, E = cnt_all.shape
    tot = cnt_all.sum(0)
    start = torch.zeros(E + 1, dtype=torch.int64)
    start[1:] = torch.cumsum((tot + 255) // 256 * 256, 0)
    chunk = max(256, _pad(-(-int(start[-1]) // R), 256))
    lo = rank * chunk
    used = max(0, min(chunk, int(start[-1]) - lo))
    send_base = (start[:E] + cnt_all[:rank].sum(0)).to(torch.int32)
    row_off = (start - lo).clamp(0, used).to(torch.int32)
    row_off[E] = used
    recv_cnt = ((start[:E] + tot - lo).clamp(0, used) - row_off[:E]).to(torch.int32)
    return send_base, row_off, recv_cnt, chunk, used


def receive_capacity(tokens: int, topk: int, n_experts: int, world: int, capacity_factor: float = 0.0) -> int:
    """Rows of one rank's receive slot (owner layout).

    Exact worst case by default: every token of every rank can send
    ``min(k, local experts)`` rows to one rank, plus up to 255 padding rows
    per local expert (expert ranges are 256-row aligned).  ``capacity_factor > 0`` caps it at that multiple of the
    mean load (``tokens * k`` rows); overflowing rows are then reported as an
    error, never silently dropped.
    """
    eloc = max(hi - lo for lo, hi in (expert_range(r, n_experts, world) for r in range(world)))
    worst = world * tokens * min(topk, eloc)
    rows = worst if capacity_factor <= 0 else min(worst, int(math.ceil(capacity_factor * tokens * topk)))
    return _pad(rows + eloc * 255, 256)


def plan_reference(cnt_all: torch.Tensor, rank: int, cap: int):
    """What ``ep_plan`` computes, in plain PyTorch (CPU oracle).

    ``cnt_all[s, e]``: rows source rank ``s`` routes to expert ``e``.  Returns
    ``(send_base [E], row_off [Eloc+1], recv_cnt [Eloc], tile_group)`` for
    ``rank``.
    """
    R, E = cnt_all.shape
    send_base = torch.zeros(E, dtype=torch.int32)
    lo, hi = expert_range(rank, E, R)
    row_off = torch.zeros(hi - lo + 1, dtype=torch.int32)
    recv_cnt = torch.zeros(hi - lo, dtype=torch.int32)
    for d in range(R):
        e0, e1 = expert_range(d, E, R)
        seg = 0
        for e in range(e0, e1):
            tot = int(cnt_all[:, e].sum())
            send_base[e] = seg + int(cnt_all[:rank, e].sum())
            if d == rank:
                row_off[e - e0] = min(seg, cap)
                recv_cnt[e - e0] = tot
            seg += _pad(tot, 256)
        if d == rank:
            row_off[e1 - e0] = min(seg, cap)
    tiles = cap // 128
    tile_group = torch.full((tiles,), -1, dtype=torch.int32)
    used = int(row_off[-1])
    for i in range(tiles):
        row = i * 128
        if row < used:
            g = max(l for l in range(hi - lo) if int(row_off[l]) <= row)
            tile_group[i] = g
    return send_base, row_off, recv_cnt, tile_group


class ExpertParallel:
    """Symmetric buffers and kernel entry points of one expert-parallel group.

    ``tokens``: rows per rank and micro-batch fed to a MoE layer (fixed for
    the life of the object: the buffers are sized for it); ``n_slots``: how
    many MoE layers keep their received activations for the backward pass.
    """

    def __init__(self, n_experts: int, topk: int, dim: int, tokens: int, n_slots: int, group=None,
                 capacity_factor: float = 0.0, timeout_s: Optional[float] = None, balanced: bool = True):
        from .symm import SymmetricHeap, heap_layout
        import torch.distributed as dist
        self.C = native()
        distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if distributed else 0
        self.world = dist.get_world_size(group) if distributed else 1
        if self.world > MAX_RANKS:
            raise ValueError(f"expert parallelism spans one box: at most {MAX_RANKS} ranks")
        if n_experts < self.world:
            raise ValueError(f"{n_experts} routed experts cannot be split over {self.world} ranks")
        if dim % 8:
            raise ValueError("model dim must be a multiple of 8 (16-byte rows)")
        self.E, self.k, self.D, self.T = n_experts, topk, dim, tokens
        self.lo, self.hi = expert_range(self.rank, n_experts, self.world)
        self.Eloc = self.hi - self.lo
        self.balanced = bool(balanced)
        # weight groups the grouped GEMMs see: all experts (balanced) or the owned ones
        self.G = n_experts if self.balanced else self.Eloc
        self.g_lo = 0 if self.balanced else self.lo
        self.cap = (balanced_capacity(tokens, topk, n_experts, self.world) if self.balanced else
                    receive_capacity(tokens, topk, n_experts, self.world, capacity_factor))
        TK = tokens * topk
        if timeout_s is None:
            timeout_s = float(os.environ.get("DSV3_EP_TIMEOUT_S", "30"))
        self.budget_ns = int(timeout_s * 1e9)
        sizes = [_FLAG_BYTES, 2 * MAX_RANKS * n_experts * 4, TK * dim * 2, TK * 4, self.cap * dim * 2]
        for _ in range(n_slots):
            sizes += [self.cap * dim * 2, self.cap * 4, self.cap * 4]
        offs = heap_layout(sizes)
        self.heap = SymmetricHeap(offs[-1], group=group)
        self.off_flags, self.off_counts, self.off_comb, self.off_dw, self.off_bwd = offs[:5]
        self.slot_offs = [tuple(offs[5 + 3 * i:8 + 3 * i]) for i in range(n_slots)]
        self.n_slots = n_slots
        dev = torch.device("cuda", self.heap.device_index)
        self.device = dev
        # local bookkeeping (not symmetric)
        self.expect = torch.zeros(5 * MAX_RANKS, dtype=torch.int32, device=dev)
        self.sendcnt = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done = torch.zeros(5, dtype=torch.int32, device=dev)
        self.peers_dev = torch.tensor(self.heap.peers, dtype=torch.int64, device=dev)
        # combine fused into the down-projection GEMM's epilogue (P2P row stores);
        # DSV3_EP_FUSED_COMBINE=0 uses the separate send-back kernel instead
        self.fused_combine = os.environ.get("DSV3_EP_FUSED_COMBINE", "1") != "0"
        self.cursor = torch.zeros(n_experts, dtype=torch.int32, device=dev)
        self.dims = [self.rank, self.world, n_experts, topk, tokens, dim, self.cap, self.budget_ns, int(self.balanced)]
        self.comb = self.heap.tensor(self.off_comb, (TK, dim), torch.bfloat16)
        self.dw_inbox = self.heap.tensor(self.off_dw, (TK,), torch.float32)
        self.slot_arange = torch.arange(TK, dtype=torch.int32, device=dev).view(tokens, topk)

    # ------------------------------------------------------------- helpers
    def offs(self, slot: int) -> List[int]:
        xs, origin, w = self.slot_offs[slot]
        return [self.off_flags, self.off_counts, self.off_comb, self.off_dw, self.off_bwd, xs, origin, w]

    def recv_rows(self, slot: int) -> torch.Tensor:
        """This rank's receive slot ``[cap, D]`` (bf16, expert-sorted rows)."""
        return self.heap.tensor(self.slot_offs[slot][0], (self.cap, self.D), torch.bfloat16)

    def recv_meta(self, slot: int):
        origin = self.heap.tensor(self.slot_offs[slot][1], (self.cap,), torch.int32)
        w = self.heap.tensor(self.slot_offs[slot][2], (self.cap,), torch.float32)
        return origin, w

    def flags(self) -> torch.Tensor:
        return self.heap.tensor(self.off_flags, (5, MAX_RANKS), torch.int32)

    # ------------------------------------------------------------- forward
    def _fork(self, overlap):
        """Run ``overlap()`` on a side stream that starts after everything
        issued so far; returns the stream (join it before using the results)."""
        if overlap is None:
            return None
        if not hasattr(self, "_side"):
            self._side = torch.cuda.Stream(device=self.device)
        cur = torch.cuda.current_stream(self.device)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            overlap()
        return self._side

    def dispatch(self, slot: int, x: torch.Tensor, idx: torch.Tensor, wts: torch.Tensor, counts: torch.Tensor,
                 overlap=None, marks=None) -> dict:
        """Plan + P2P dispatch of ``x [T, D]`` along ``idx [T, k]``; waits for
        every peer's rows.  Returns the receive-side plan.  ``overlap()``
        (independent work, e.g. the shared experts) runs on a side stream
        while the rows are in flight; ``plan["side"]`` must be joined."""
        C, dev = self.C, self.device
        plan = {
            "cnt_all": torch.empty(self.world, self.E, dtype=torch.int32, device=dev),
            "send_base": torch.empty(self.E, dtype=torch.int32, device=dev),
            "row_off": torch.empty(self.G + 1, dtype=torch.int32, device=dev),
            "recv_cnt": torch.empty(self.G, dtype=torch.int32, device=dev),
            "tile_group": torch.empty(self.cap // 128, dtype=torch.int32, device=dev),
            "route": torch.empty(2, self.T * self.k, dtype=torch.int32, device=dev),
            "bal_info": torch.zeros(4, dtype=torch.int32, device=dev),
        }
        offs = self.offs(slot)
        bal = plan["bal_info"] if self.balanced else None
        C.ep_plan(self.heap.peers, offs, self.dims, counts, self.expect, self.sendcnt, plan["cnt_all"],
                  plan["send_base"], plan["row_off"], plan["recv_cnt"], plan["tile_group"], self.cursor, bal)
        C.ep_dispatch(self.heap.peers, offs, self.dims, x, idx, wts, plan["send_base"], self.cursor, plan["route"],
                      plan["row_off"], plan["recv_cnt"], self.done[0:1], bal)
        plan["side"] = self._fork(overlap)
        if marks is not None:
            marks("ep plan+send")
        C.ep_wait(self.heap.peers, offs, self.dims, PH_DISPATCH, self.expect)
        return plan

    def combine_send(self, slot: int, rows: torch.Tensor, row_off: torch.Tensor) -> None:
        """Expert outputs ``rows [cap, D]`` back to the home ranks; waits for ours."""
        offs = self.offs(slot)
        self.C.ep_send_back(self.heap.peers, offs, self.dims, PH_COMBINE, rows, None, row_off, self.done[1:2])
        self.C.ep_wait(self.heap.peers, offs, self.dims, PH_COMBINE, self.expect)

    # ------------------------------------------------------------ backward
    def dispatch_bwd(self, slot: int, g: torch.Tensor, route: torch.Tensor, overlap=None, marks=None):
        offs = self.offs(slot)
        self.C.ep_dispatch_bwd(self.heap.peers, offs, self.dims, g, route, self.done[2:3])
        side = self._fork(overlap)
        if marks is not None:
            marks("ep send bwd")
        self.C.ep_wait(self.heap.peers, offs, self.dims, PH_BWD_DISPATCH, self.expect)
        return side

    def bwd_prep(self, slot: int, ys: torch.Tensor, row_off: torch.Tensor, dys: torch.Tensor,
                 dw_rows: torch.Tensor) -> None:
        self.C.ep_bwd_prep(self.heap.peers, self.offs(slot), self.dims, ys, row_off, dys, dw_rows)

    def combine_send_bwd(self, slot: int, rows: torch.Tensor, dw_rows: torch.Tensor, row_off: torch.Tensor) -> None:
        offs = self.offs(slot)
        self.C.ep_send_back(self.heap.peers, offs, self.dims, PH_BWD_COMBINE, rows, dw_rows, row_off,
                            self.done[3:4])
        self.C.ep_wait(self.heap.peers, offs, self.dims, PH_BWD_COMBINE, self.expect)

    def close(self) -> None:
        self.heap.close()


def _no_mark(name: str) -> None:
    return None


def moe_forward_ep(ep: ExpertParallel, slot: int, xn: torch.Tensor, idx, wts, counts, w13_local, w2_local,
                   out: torch.Tensor, inter_dim: int, marks=_no_mark, overlap=None) -> dict:
    """Routed-expert part of a MoE layer under expert parallelism.

    ``w13_local [G, 2, I, D]`` / ``w2_local [G, D, I]``: the bf16 weights of
    the layout's weight groups (``ep.G``: every expert in the balanced
    layout, the owned ones in the owner layout).  Adds ``sum_j w[t, j] * expert_j(x[t])`` into the
    fp32 ``out``.  Returns the context the backward needs.  ``marks(name)``
    is called after each phase (the microbenchmark records events there);
    ``overlap()`` runs on a side stream during the transfers and is joined
    before the combine touches ``out``.
    """
    C = ep.C
    plan = ep.dispatch(slot, xn, idx, wts, counts, overlap=overlap, marks=marks)
    marks("ep dispatch wait")
    xs = ep.recv_rows(slot)
    h = torch.empty(ep.cap, inter_dim, dtype=torch.bfloat16, device=xn.device)
    gu = torch.empty(ep.cap, 2 * inter_dim, dtype=torch.bfloat16, device=xn.device)
    C.swiglu_fwd(xs, w13_local, plan["tile_group"], h, gu, group_rows=256)
    marks("experts gate/up fwd")
    ys = torch.empty(ep.cap, ep.D, dtype=torch.bfloat16, device=xn.device)
    if ep.fused_combine:
        # down projection whose epilogue stores every row into its home rank's
        # combine inbox; the last CTA raises the combine flag on every rank
        origin, _ = ep.recv_meta(slot)
        C.grouped_scatter(h, w2_local, False, plan["tile_group"], ys, 256, ep.peers_dev, ep.off_comb, origin, None,
                          0, ep.T * ep.k, ep.off_flags, ep.rank, PH_COMBINE, ep.done[4:5])
        marks("experts fwd")
        C.ep_wait(ep.heap.peers, ep.offs(slot), ep.dims, PH_COMBINE, ep.expect)
    else:
        C.grouped_fwd(h, w2_local, plan["tile_group"], ys, group_rows=256)
        marks("experts fwd")
        ep.combine_send(slot, ys, plan["row_off"])
    marks("ep combine wait")
    side = plan.pop("side")
    if side is not None:
        torch.cuda.current_stream(xn.device).wait_stream(side)
    marks("shared experts join")
    C.combine_fwd(ep.comb, ep.slot_arange, wts, out)
    marks("combine fwd")
    plan.update(slot=slot, xs=xs, h=h, gu=gu, ys=ys)
    return plan


def moe_backward_ep(ep: ExpertParallel, ctx: dict, dout_bf16: torch.Tensor, w13_local, w2_local, g13_local,
                    g2_local, dx_acc: torch.Tensor, inter_dim: int, marks=_no_mark, overlap=None) -> torch.Tensor:
    """Backward of ``moe_forward_ep``: accumulates expert weight gradients of
    the owned experts into ``g13_local [Eloc, 2I, D]`` / ``g2_local [Eloc, D, I]``,
    adds the token input gradients into ``dx_acc`` (fp32) and returns the
    gate-weight gradients ``dw [T, k]`` (fp32, home side).  ``overlap()`` runs
    on a side stream during the transfers, joined before ``dx_acc`` is read."""
    C = ep.C
    slot = ctx["slot"]
    side = ep.dispatch_bwd(slot, dout_bf16, ctx["route"], overlap=overlap, marks=marks)
    marks("ep dispatch wait bwd")
    dys = torch.empty(ep.cap, ep.D, dtype=torch.bfloat16, device=dout_bf16.device)
    dw_rows = torch.empty(ep.cap, dtype=torch.float32, device=dout_bf16.device)
    ep.bwd_prep(slot, ctx["ys"], ctx["row_off"], dys, dw_rows)
    marks("ep bwd prep")
    dgu = torch.empty(ep.cap, 2 * inter_dim, dtype=torch.bfloat16, device=dout_bf16.device)
    C.swiglu_dgrad(dys, w2_local, ctx["tile_group"], ctx["gu"], dgu, group_rows=256)
    marks("experts swiglu dgrad")
    C.grouped_wgrad(dys, ctx["h"], ctx["row_off"], g2_local)
    marks("experts down wgrad")
    dxs = torch.empty(ep.cap, ep.D, dtype=torch.bfloat16, device=dout_bf16.device)
    w13_2d = w13_local.reshape(ep.G, 2 * inter_dim, ep.D)
    if ep.fused_combine:
        # input-gradient GEMM whose epilogue sends each row (and its gate-weight
        # gradient) to the home rank; the weight gradient runs meanwhile
        origin, _ = ep.recv_meta(slot)
        C.grouped_scatter(dgu, w13_2d, True, ctx["tile_group"], dxs, 256, ep.peers_dev, ep.off_comb, origin, dw_rows,
                          ep.off_dw, ep.T * ep.k, ep.off_flags, ep.rank, PH_BWD_COMBINE, ep.done[4:5])
        marks("experts dgrad+send")
        C.grouped_wgrad(dgu, ctx["xs"], ctx["row_off"], g13_local)
        marks("experts bwd")
        C.ep_wait(ep.heap.peers, ep.offs(slot), ep.dims, PH_BWD_COMBINE, ep.expect)
    else:
        C.grouped_dgrad(dgu, w13_2d, ctx["tile_group"], dxs, group_rows=256)
        C.grouped_wgrad(dgu, ctx["xs"], ctx["row_off"], g13_local)
        marks("experts bwd")
        ep.combine_send_bwd(slot, dxs, dw_rows, ctx["row_off"])
    marks("ep combine wait bwd")
    if side is not None:
        torch.cuda.current_stream(dx_acc.device).wait_stream(side)
    marks("shared experts join")
    C.unpermute_bwd(ep.comb, ep.slot_arange, dx_acc)
    marks("combine bwd")
    return ep.dw_inbox.view(ep.T, ep.k)
