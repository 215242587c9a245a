"""The B200 training engine: explicit forward and backward of the whole model
(Transformer + MTP + fused LM-head cross-entropy) on the sm_100a kernels.

There is no autograd and no tracing compiler in the step.  Each layer's
forward saves exactly what its backward needs; the backward walks the layers
in reverse, accumulating weight gradients straight into the fp32 flat gradient
buffers (``ops.flat``) with the weight-gradient GEMM epilogues.  The residual
stream and its gradient are fp32 (as the reference's autocast run keeps them:
embedding output and residual adds are fp32 there too); every GEMM operand is
bf16 with fp32 accumulation in TMEM.

Per micro-batch the kernel sequence is (``L`` layers, ``T = B * S`` tokens):

forward, per layer
  RMSNorm -> q / kv_a projections (tcgen05 GEMM) -> latent RMSNorm -> kv_b
  projection -> Q/K/V packing with RoPE -> flash attention -> o-projection
  accumulated into the fp32 residual (GEMM epilogue) -> RMSNorm ->
  dense SwiGLU (fused gate/up GEMM + SwiGLU epilogue, down GEMM into the
  residual) or MoE (router GEMM -> top-k kernel -> padded expert permutation
  -> gather -> grouped SwiGLU GEMM -> grouped down GEMM -> weighted combine
  into the residual, plus the shared expert)
head
  final RMSNorm, MTP block (same kernels), one fused LM-head + CE pass over
  main and MTP rows (no logits in memory), log-sum-exp combine, per-segment
  mean.
backward
  CE gradient GEMM (chunked dlogits) -> MTP backward -> final-norm backward ->
  layers in reverse -> embedding scatter-add.

Semantics follow the reference model exactly (see ``models/``); the loss and
gradients are checked against the eager PyTorch model in the GPU tests.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from . import _ext
from ._ext import native, check_status
from .flat import FlatAdamW, FlatParams
from .rope import rope_cos_sin

BF16 = torch.bfloat16
F32 = torch.float32


def _pad(n: int, m: int) -> int:
    return (n + m - 1) // m * m


class PhaseTimer:
    """Device time per named phase of the training step.

    ``mark(name)`` records a CUDA event on the current stream; the time since
    the previous mark is booked to ``name``.  While a CUDA graph is being
    captured the events become event-record nodes of the graph
    (``external=True``), so a replay re-records them and the phases of the
    graphed micro-step are timed without host launch gaps in between.
    ``book(events)`` synchronises and adds a list of marks' intervals to
    ``totals`` (ms); ``collect()`` books the marks recorded since the last
    ``take()``.
    """

    def __init__(self, device):
        self.device = device
        self.totals: Dict[str, float] = {}
        self._events: list = []

    def mark(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True, external=bool(torch.cuda.is_current_stream_capturing()))
        ev.record()
        self._events.append((name, ev))

    def take(self) -> list:
        ev, self._events = self._events, []
        return ev

    def book(self, events: list) -> None:
        torch.cuda.synchronize(self.device)
        for (_, a), (name, b) in zip(events, events[1:]):
            self.totals[name] = self.totals.get(name, 0.0) + a.elapsed_time(b)

    def collect(self) -> Dict[str, float]:
        self.book(self.take())
        return self.totals


class _Ctx(dict):
    """Saved tensors of one layer for its backward."""
    __getattr__ = dict.__getitem__
    __setattr__ = dict.__setitem__


class TrainEngine:
    """Fused forward/backward + optimizer for ``Transformer`` (+ MTP) on one GPU
    (one rank of a data-parallel job when ``torch.distributed`` is up)."""

    def __init__(self, model, mtp_wrapper, config, groups, dp_group=None):
        self.model = model
        self.mtp = mtp_wrapper
        self.config = config
        self.cfg = model.config
        self.device = next(model.parameters()).device
        self.C = native()
        c = self.cfg
        self.D = c["dim"]
        self.H = c["n_heads"]
        self.dn, self.dr, self.dv = c["qk_nope_head_dim"], c["qk_rope_head_dim"], c["v_head_dim"]
        self.R = c["kv_lora_rank"]
        self.DP = max(32, _pad(self.dn + self.dr, 16))
        self.V = c["vocab_size"]
        self.Vp = _pad(self.V, 64)
        # LoRA query path wq_a -> q_norm -> wq_b (reference models/mla.py:43-46, :105-108)
        self.q_lora = int(c.get("q_lora_rank", 0) or 0)
        if self.q_lora > 0 and self.q_lora % 8:
            raise ValueError("q_lora_rank must be a multiple of 8 (16-byte GEMM rows)")
        self.max_seq_len = c["max_seq_len"]
        self.ce_chunk = int(os.environ.get("DSV3_CE_CHUNK_ROWS", "16384"))
        dist_on = torch.distributed.is_available() and torch.distributed.is_initialized()
        # data parallel step over peer memory (reduce-scatter + sharded AdamW +
        # all-gather, csrc/dp.cu); DSV3_DP_NCCL=1 selects NCCL all-reduce instead
        self._fused_dp = (dist_on and torch.distributed.get_world_size(dp_group) > 1
                          and os.environ.get("DSV3_DP_NCCL", "0") != "1")
        # Routed experts sharded over the expert-parallel ranks: each rank
        # keeps weights, gradients and optimizer state of its own experts only.
        world0 = torch.distributed.get_world_size(dp_group) if dist_on else 1
        rank0 = torch.distributed.get_rank(dp_group) if dist_on else 0
        ep_size0 = int(getattr(config, "ep_size", 1))
        self.shard_experts = (dist_on and world0 > 1 and ep_size0 != 1
                              and bool(getattr(config, "ep_shard_experts", False)))
        if self.shard_experts:
            from parallel.ep import expert_range
            self._exp_range = expert_range(rank0, c["n_routed_experts"], world0)
        self._build_flat(groups)
        if self.shard_experts:
            ids = {id(p) for p in self.flat_expert.params}
            self._local_expert_named = [(n, p) for n, p in model.named_parameters() if id(p) in ids]
        self.optimizer = FlatAdamW(groups, self.flats, lr=config.lr, betas=(config.beta1, config.beta2),
                                   flat_groups=[0, 1, 0][:len(self.flats)])
        cos, sin = rope_cos_sin(self.max_seq_len, self.dr, float(c["rope_theta"]), self.device)
        self.cos, self.sin = cos, sin
        self.world_size = 1
        self.rank = 0
        self.dp = None
        if dist_on:
            from parallel.dp import DataParallel, FusedDataParallel
            self.dp = (FusedDataParallel(self, self.dp_heap, group=dp_group) if self._fused_dp
                       else DataParallel(self, group=dp_group))
            self.world_size = self.dp.world_size
            self.rank = self.dp.rank
        # Expert parallelism: routed experts spread over the data-parallel
        # ranks, tokens moved by the peer-memory kernels of parallel/ep.py.
        self.ep = None
        self.ep_size = int(getattr(config, "ep_size", 1))
        if self.ep_size not in (0, 1) and self.ep_size != self.world_size:
            raise NotImplementedError("the expert-parallel group spans all ranks (ep_size 0 or the world size)")
        self.use_ep = self.dp is not None and self.world_size > 1 and self.ep_size != 1
        self._moe_slot = {id(mod): i for i, mod in enumerate(model.moe_layers())}
        self._last_losses: Optional[torch.Tensor] = None
        self._finite = torch.ones(1, dtype=torch.bool, device=self.device)
        self._segcache: Dict[tuple, tuple] = {}
        self._graphs: Dict[tuple, tuple] = {}
        # Capture the micro-step in a CUDA graph (DSV3_CUDA_GRAPH=0 turns it off).
        self.use_graphs = os.environ.get("DSV3_CUDA_GRAPH", "1") == "1"
        # NVTX ranges per layer / phase for timeline tools (DSV3_NVTX=1)
        self.nvtx = os.environ.get("DSV3_NVTX", "0") == "1"
        # per-phase device timing (set by the benchmark's breakdown step)
        self.phase_timer: Optional[PhaseTimer] = None
        # Activation recomputation: keep only each layer's input and rerun the
        # layer's forward in the backward pass (config.activation_recompute or
        # DSV3_RECOMPUTE=1).  Off by default: on 180 GB the memory is better
        # spent on larger micro-batches; it lets long sequences or the scaled
        # model fit.
        self.recompute = bool(getattr(config, "activation_recompute", False)) or \
            os.environ.get("DSV3_RECOMPUTE", "0") == "1"
        # MoE layers: the FFN norm's backward runs fused with the sum of the
        # shared, routed and router input gradients (DSV3_MOE_NORM_FUSED=0: the
        # separate un-permute, router data-gradient GEMM and norm backward)
        self.fuse_moe_norm = os.environ.get("DSV3_MOE_NORM_FUSED", "1") != "0"

    def _mark(self, name: str) -> None:
        if self.phase_timer is not None:
            self.phase_timer.mark(name)

    # ---------------------------------------------------------------- layout
    def _build_flat(self, groups) -> None:
        """Pack parameters into contiguous blocks the kernels can address.

        SwiGLU weights get dedicated blocks ([w1, w3] per expert, then all
        w2) so the grouped GEMMs see ``[E, 2, I, D]`` and ``[E, D, I]``
        operands; every other decayed tensor is its own block.  Undecayed
        (1-D) parameters live in a second buffer.
        """
        m = self.model
        blocks: List[List[torch.nn.Parameter]] = []
        placed = set()

        def add(block):
            block = [p for p in block if id(p) not in placed]
            for p in block:
                placed.add(id(p))
            if block:
                blocks.append(block)

        expert_blocks: List[List[torch.nn.Parameter]] = []
        remote: List[torch.nn.Parameter] = []
        for layer in m.layers:
            # q (or LoRA q_a) and kv_a projections share their input: one
            # [wq; wkv_a] block makes them one GEMM (and one data-gradient, one
            # weight-gradient)
            add([self._q_in(layer.attn), layer.attn.wkv_a.weight])
            ffn = layer.ffn
            if hasattr(ffn, "experts") and self.shard_experts:
                lo, hi = self._exp_range
                local = list(ffn.experts[lo:hi])
                expert_blocks.append([w for e in local for w in (e.w1.weight, e.w3.weight)])
                expert_blocks.append([e.w2.weight for e in local])
                for e in list(ffn.experts[:lo]) + list(ffn.experts[hi:]):
                    for p in (e.w1.weight, e.w2.weight, e.w3.weight):
                        # other ranks own these: drop the storage before the
                        # flat buffers are allocated (lower peak memory)
                        p.data = torch.empty(0, dtype=p.dtype, device=p.device)
                        p.grad = None
                        remote.append(p)
                for p in [w for b in expert_blocks[-2:] for w in b] + remote:
                    placed.add(id(p))
                for e in ffn.shared_experts:
                    add([e.w1.weight, e.w3.weight])
                    add([e.w2.weight])
            elif hasattr(ffn, "experts"):
                add([w for e in ffn.experts for w in (e.w1.weight, e.w3.weight)])
                add([e.w2.weight for e in ffn.experts])
                for e in ffn.shared_experts:
                    add([e.w1.weight, e.w3.weight])
                    add([e.w2.weight])
            else:
                add([ffn.w1.weight, ffn.w3.weight])
                add([ffn.w2.weight])
        if self.mtp is not None:
            for mod in self.mtp.mtp_modules:
                add([mod.block.w1.weight, mod.block.w3.weight])
                add([mod.block.w2.weight])
        for p in groups[0]["params"]:
            add([p])
        decay_ids = {id(p) for p in groups[0]["params"]}
        if any(id(p) not in decay_ids for b in blocks + expert_blocks for p in b):
            raise RuntimeError("a packed block contains an undecayed parameter")
        nodecay_blocks = [[p] for p in groups[1]["params"]]
        alloc_d = alloc_n = None
        self.dp_heap = None
        if self._fused_dp:
            # flat buffers in a symmetric heap: the data-parallel step reads the
            # peers' gradients and writes the peers' weights directly
            from parallel.dp import FusedDataParallel
            self.dp_heap, alloc_d, alloc_n = FusedDataParallel.make_heap(
                [FlatParams.layout_numel(blocks), FlatParams.layout_numel(nodecay_blocks)])
        self.flat_decay = FlatParams(blocks, self.device, alloc=alloc_d)
        self.flat_nodecay = FlatParams(nodecay_blocks, self.device, alloc=alloc_n)
        self.flats = [self.flat_decay, self.flat_nodecay]
        self.flat_expert = None
        if self.shard_experts:
            # this rank's routed experts: local memory, never averaged over ranks
            self.flat_expert = FlatParams(expert_blocks, self.device)
            self.flat_expert.rank_local = True
            self.flats.append(self.flat_expert)
            self._remote_experts = remote

    def _fl(self, p) -> FlatParams:
        if id(p) in self.flat_decay.offsets:
            return self.flat_decay
        if self.flat_expert is not None and id(p) in self.flat_expert.offsets:
            return self.flat_expert
        return self.flat_nodecay

    def _local_experts(self, moe, ep):
        """bf16 weights and fp32 gradient views of the expert-parallel layout's
        weight groups: (w13 [G, 2, I, D], w2 [G, D, I], g13 [G, 2I, D],
        g2 [G, D, I]); every expert in the balanced layout, this rank's own
        in the owner layout."""
        E = moe.n_routed_experts
        if ep.balanced:
            w1, w2 = moe.experts[0].w1.weight, moe.experts[0].w2.weight
            return (self.swiglu_w13(w1, E), self.stacked(w2, E), self.swiglu_g13(w1, E), self.stacked(w2, E, grad=True))
        if self.shard_experts:
            first = moe.experts[ep.lo]
            n = ep.hi - ep.lo
            return (self.swiglu_w13(first.w1.weight, n), self.stacked(first.w2.weight, n),
                    self.swiglu_g13(first.w1.weight, n), self.stacked(first.w2.weight, n, grad=True))
        w1, w2 = moe.experts[0].w1.weight, moe.experts[0].w2.weight
        return (self.swiglu_w13(w1, E)[ep.lo:ep.hi], self.stacked(w2, E)[ep.lo:ep.hi],
                self.swiglu_g13(w1, E)[ep.lo:ep.hi], self.stacked(w2, E, grad=True)[ep.lo:ep.hi])

    def w(self, p) -> torch.Tensor:
        """bf16 shadow of parameter ``p``."""
        return self._fl(p).view(self._fl(p).shadow, p)

    def g(self, p) -> torch.Tensor:
        """fp32 gradient buffer of parameter ``p``."""
        return self._fl(p).view(self._fl(p).grad, p)

    def f32(self, p) -> torch.Tensor:
        return self._fl(p).view(self._fl(p).master, p)

    def swiglu_w13(self, w1, n_groups: int) -> torch.Tensor:
        I, D = w1.shape
        fl = self._fl(w1)
        return fl.block_view(fl.shadow, w1, (n_groups, 2, I, D))

    def swiglu_g13(self, w1, n_groups: int) -> torch.Tensor:
        I, D = w1.shape
        fl = self._fl(w1)
        return fl.block_view(fl.grad, w1, (n_groups, 2 * I, D))

    def stacked(self, w, n_groups: int, grad: bool = False) -> torch.Tensor:
        fl = self._fl(w)
        return fl.block_view(fl.grad if grad else fl.shadow, w, (n_groups,) + tuple(w.shape))

    @staticmethod
    def _q_in(attn):
        """The query projection applied to the normalised input: ``wq``, or ``wq_a`` of the LoRA chain."""
        return attn.wq_a.weight if getattr(attn, "q_lora_rank", 0) > 0 else attn.wq.weight

    def qkva_block(self, attn, grad: bool = False) -> torch.Tensor:
        """``[wq; wkv_a]`` (``[wq_a; wkv_a]`` with LoRA q) as one ``[Nq_in + R + dr, D]`` operand (shadow or grad)."""
        first = self._q_in(attn)
        fl = self._fl(first)
        rows = first.shape[0] + attn.wkv_a.weight.shape[0]
        return fl.block_view(fl.grad if grad else fl.shadow, first, (rows, self.D))

    # --------------------------------------------------------------- helpers
    def _norm(self, x, weight_param, eps=1e-6):
        T = x.shape[0]
        y = torch.empty(T, x.shape[1], dtype=BF16, device=self.device)
        r = torch.empty(T, dtype=F32, device=self.device)
        self.C.rmsnorm_fwd(x, self.f32(weight_param), eps, y, r)
        return y, r

    def _linear(self, x, p, out_dtype=BF16):
        y = torch.empty(x.shape[0], p.shape[0], dtype=out_dtype, device=self.device)
        self.C.linear_fwd(x, self.w(p), y, False)
        return y

    def _linear_bwd(self, dy, x, p, dx_acc=None, accumulate=True):
        """dW += dy^T x; returns dx (bf16) unless ``dx_acc`` (fp32) is given,
        which is accumulated into (or overwritten when ``accumulate`` is False)."""
        self.C.linear_wgrad(dy, x, self.g(p))
        if dx_acc is not None:
            self.C.linear_dgrad(dy, self.w(p), dx_acc, accumulate)
            return dx_acc
        dx = torch.empty(dy.shape[0], p.shape[1], dtype=BF16, device=self.device)
        self.C.linear_dgrad(dy, self.w(p), dx)
        return dx

    # ------------------------------------------------------------ attention
    def _mla_fwd(self, attn, xn, B, S):
        C, H, dn, dr, dv, R = self.C, self.H, self.dn, self.dr, self.dv, self.R
        T = B * S
        ctx = _Ctx(xn=xn)
        Nq = H * (dn + dr)
        nq_in = self.q_lora or Nq
        wqa = self.qkva_block(attn)
        qkva = torch.empty(T, wqa.shape[0], dtype=BF16, device=self.device)
        C.linear_fwd(xn, wqa, qkva)                                   # [T, nq_in + R + dr]
        kv_a = qkva[:, nq_in:]
        if self.q_lora:
            qn = torch.empty(T, self.q_lora, dtype=BF16, device=self.device)
            rq = torch.empty(T, dtype=F32, device=self.device)
            C.rmsnorm_fwd(qkva[:, :nq_in], self.f32(attn.q_norm.weight), 1e-6, qn, rq)
            q = self._linear(qn, attn.wq_b.weight)                    # [T, H*(dn+dr)]
            ctx.update(qa=qkva[:, :nq_in], qn=qn, rq=rq)
        else:
            q = qkva[:, :Nq]
        lat = torch.empty(T, R, dtype=BF16, device=self.device)
        rkv = torch.empty(T, dtype=F32, device=self.device)
        C.rmsnorm_fwd(kv_a[:, :R], self.f32(attn.kv_norm.weight), 1e-6, lat, rkv)
        kvb = self._linear(lat, attn.wkv_b.weight)                    # [T, H*(dn+dv)]
        Q = torch.empty(B * H, S, self.DP, dtype=BF16, device=self.device)
        K = torch.empty_like(Q)
        Vt = torch.empty(B * H, S, dv, dtype=BF16, device=self.device)
        C.mla_pack(q, kvb, kv_a[:, R:], Q, K, Vt, B, S, H, dn, dr, dv, self.cos, self.sin, 0)
        O = torch.empty(T, H * dv, dtype=BF16, device=self.device)
        L = torch.empty(B * H, S, dtype=F32, device=self.device)
        self._mark("attn proj fwd")
        C.flash_fwd(Q, K, Vt, O, L, 0, attn.softmax_scale, True, H)
        self._mark("flash fwd")
        ctx.update(kv_a=kv_a, lat=lat, rkv=rkv, Q=Q, K=K, V=Vt, O=O, L=L)
        return ctx

    def _mla_bwd(self, attn, ctx, dres_bf16, dxn_acc, B, S):
        """dres_bf16: gradient of the o-projection output.  Accumulates into dxn_acc (fp32)."""
        C, H, dn, dr, dv, R = self.C, self.H, self.dn, self.dr, self.dv, self.R
        T = B * S
        dO = self._linear_bwd(dres_bf16, ctx.O, attn.wo.weight)       # [T, H*dv]
        dQ = torch.zeros(B * H, S, self.DP, dtype=F32, device=self.device)
        dK = torch.empty_like(dQ)
        dV = torch.empty(B * H, S, dv, dtype=F32, device=self.device)
        delta = torch.empty(B * H, S, dtype=F32, device=self.device)
        self._mark("o-proj bwd")
        C.flash_bwd(ctx.Q, ctx.K, ctx.V, ctx.O, dO, ctx.L, delta, dQ, dK, dV, 0, attn.softmax_scale, True, H)
        self._mark("flash bwd")
        Nq = H * (dn + dr)
        nq_in = self.q_lora or Nq
        dqkva = torch.empty(T, nq_in + R + dr, dtype=BF16, device=self.device)
        dkv_a = dqkva[:, nq_in:]
        dq = torch.empty(T, Nq, dtype=BF16, device=self.device) if self.q_lora else dqkva[:, :Nq]
        dkvb = torch.empty(T, H * (dn + dv), dtype=BF16, device=self.device)
        C.mla_unpack(dQ, dK, dV, dq, dkvb, dkv_a[:, R:], B, S, H, dn, dr, dv, self.cos, self.sin, 0)
        dlat = self._linear_bwd(dkvb, ctx.lat, attn.wkv_b.weight)
        C.rmsnorm_bwd(dlat, ctx.kv_a[:, :R], self.f32(attn.kv_norm.weight), ctx.rkv, None, dkv_a[:, :R], None,
                      self.g(attn.kv_norm.weight))
        if self.q_lora:
            dqn = self._linear_bwd(dq, ctx.qn, attn.wq_b.weight)      # [T, q_lora], dW(wq_b) accumulated
            C.rmsnorm_bwd(dqn, ctx.qa, self.f32(attn.q_norm.weight), ctx.rq, None, dqkva[:, :nq_in], None,
                          self.g(attn.q_norm.weight))
        C.linear_wgrad(dqkva, ctx.xn, self.qkva_block(attn, grad=True))
        C.linear_dgrad(dqkva, self.qkva_block(attn), dxn_acc, False)
        self._mark("attn proj bwd")

    # ------------------------------------------------------------------ FFN
    def _swiglu_dense_fwd(self, w1, w2, xn, out, resid_in=None):
        """out += w2(silu(w1 x) * w3 x) (or out = resid_in + ...) with one fused gate/up GEMM."""
        T = xn.shape[0]
        I = w1.shape[0]
        h = torch.empty(T, I, dtype=BF16, device=self.device)
        gu = torch.empty(T, 2 * I, dtype=BF16, device=self.device)
        self.C.swiglu_fwd(xn, self.swiglu_w13(w1, 1), self._empty_i32, h, gu)
        self.C.linear_fwd(h, self.w(w2), out, True, resid_in)
        return _Ctx(h=h, gu=gu)

    def _swiglu_dense_bwd(self, w1, w2, ctx, xn, dres_bf16, dxn_acc, accumulate=True):
        I = w1.shape[0]
        T = xn.shape[0]
        dgu = torch.empty(T, 2 * I, dtype=BF16, device=self.device)
        self.C.swiglu_dgrad(dres_bf16, self.stacked(w2, 1), self._empty_i32, ctx.gu, dgu)
        self.C.linear_wgrad(dres_bf16, ctx.h, self.g(w2))
        w13 = self.swiglu_w13(w1, 1).view(2 * I, -1)
        self.C.linear_dgrad(dgu, w13, dxn_acc, accumulate)
        self.C.linear_wgrad(dgu, xn, self.swiglu_g13(w1, 1).view(2 * I, -1))

    def _fork(self, work):
        """Run ``work()`` on the engine's side stream, ordered after everything
        issued so far on the current stream; returns the stream to join."""
        if not hasattr(self, "_side_stream"):
            self._side_stream = torch.cuda.Stream(device=self.device)
        cur = torch.cuda.current_stream(self.device)
        self._side_stream.wait_stream(cur)
        with torch.cuda.stream(self._side_stream):
            work()
        return self._side_stream

    def _join(self, side) -> None:
        if side is not None:
            torch.cuda.current_stream(self.device).wait_stream(side)

    def _ep_group(self, tokens: int):
        """The expert-parallel buffers, created on first use (a collective:
        every rank reaches it at the same MoE layer)."""
        if self.ep is None:
            from parallel.ep import ExpertParallel
            c = self.cfg
            # balanced layout while expert weights are replicated (DSV3_EP_BALANCED=0: owner layout)
            balanced = not self.shard_experts and os.environ.get("DSV3_EP_BALANCED", "1") != "0"
            self.ep = ExpertParallel(c["n_routed_experts"], c["n_activated_experts"], self.D, tokens,
                                     n_slots=len(self._moe_slot), group=self.dp.group,
                                     capacity_factor=float(getattr(self.config, "ep_capacity_factor", 0.0)),
                                     balanced=balanced)
        if self.ep.T != tokens:
            raise RuntimeError(f"expert-parallel buffers are sized for {self.ep.T} tokens per micro-batch, got "
                               f"{tokens}; keep the micro-batch shape fixed")
        return self.ep

    def _router(self, moe, xn):
        C = self.C
        T = xn.shape[0]
        E, k = moe.n_routed_experts, moe.topk
        Ep = _pad(E, 8)
        logits = torch.empty(T, Ep, dtype=F32, device=self.device)
        C.linear_fwd(xn, self.w(moe.gate.weight), logits[:, :E], False)
        idx = torch.empty(T, k, dtype=torch.int32, device=self.device)
        wts = torch.empty(T, k, dtype=F32, device=self.device)
        ssel = torch.empty(T, k, dtype=F32, device=self.device)
        counts = torch.zeros(E, dtype=torch.int32, device=self.device)
        C.router_topk(logits, moe.gate.bias, E, k, float(moe.gate.route_scale), idx, wts, ssel, counts)
        moe._last_indices = idx
        moe._last_weights = wts
        moe._last_counts = counts
        return idx, wts, ssel, counts, Ep

    def _moe_fwd_ep(self, moe, xn, resid_in):
        from parallel.ep import moe_forward_ep
        T = xn.shape[0]
        E, I = moe.n_routed_experts, moe.moe_inter_dim
        ep = self._ep_group(T)
        idx, wts, ssel, counts, Ep = self._router(moe, xn)
        out = torch.empty_like(resid_in) if moe.shared_experts else resid_in.clone()
        shared = []

        def shared_fwd():   # overlaps the dispatch (side stream, joined before the combine)
            for i, e in enumerate(moe.shared_experts):
                shared.append(self._swiglu_dense_fwd(e.w1.weight, e.w2.weight, xn, out, resid_in if i == 0 else None))
        w13, w2, _, _ = self._local_experts(moe, ep)
        self._mark("router fwd")
        ectx = moe_forward_ep(ep, self._moe_slot[id(moe)], xn, idx, wts, counts, w13, w2, out, I,
                              marks=self._mark, overlap=shared_fwd if moe.shared_experts else None)
        return _Ctx(ep=ectx, idx=idx, wts=wts, ssel=ssel, shared=shared, Ep=Ep, counts=counts), out

    def _moe_bwd_ep(self, moe, ctx, xn, dres_bf16, dxn_acc, norm=None):
        from parallel.ep import moe_backward_ep
        C, ep = self.C, self.ep
        E, I = moe.n_routed_experts, moe.moe_inter_dim
        if not moe.shared_experts:
            dxn_acc.zero_()

        def shared_bwd():   # overlaps the gradient dispatch (joined before dxn_acc is summed into)
            for i, (e, sctx) in enumerate(zip(moe.shared_experts, ctx.shared)):
                self._swiglu_dense_bwd(e.w1.weight, e.w2.weight, sctx, xn, dres_bf16, dxn_acc, accumulate=i > 0)
        w13, w2, g13, g2 = self._local_experts(moe, ep)
        dw = moe_backward_ep(ep, ctx.ep, dres_bf16, w13, w2, g13, g2, dxn_acc, I, marks=self._mark,
                             overlap=shared_bwd if moe.shared_experts else None)
        if self._norm_fusable(moe, norm):
            dlog = self._router_dlog(moe, ctx, xn, dw)
            self._moe_norm_bwd(moe, None, None, dxn_acc, dlog, norm)
            self._mark("router bwd + norm bwd")
            return True
        self._router_bwd(moe, ctx, xn, dw, dxn_acc)
        self._mark("router bwd")
        return False

    def _router_dlog(self, moe, ctx, xn, dw):
        """Router logit gradients [T, Ep] (bf16) and the gate weight gradient."""
        C = self.C
        T, E = xn.shape[0], moe.n_routed_experts
        dlog = torch.empty(T, ctx.Ep, dtype=BF16, device=self.device)
        C.router_bwd(dw, ctx.ssel, ctx.idx, float(moe.gate.route_scale), dlog)
        C.linear_wgrad(dlog[:, :E], xn, self.g(moe.gate.weight))
        return dlog

    def _router_bwd(self, moe, ctx, xn, dw, dxn_acc):
        dlog = self._router_dlog(moe, ctx, xn, dw)
        self.C.linear_dgrad(dlog[:, :moe.n_routed_experts], self.w(moe.gate.weight), dxn_acc)

    def _norm_fusable(self, moe, norm):
        """Whether the FFN norm's backward can run fused with the MoE input-gradient sum."""
        if norm is None or not self.fuse_moe_norm:
            return False
        D = self.D
        return D % 64 == 0 and D // 64 in (1, 2, 3, 4, 6, 8, 12, 16, 24, 32) and \
            self.C.moe_norm_bwd_smem(moe.n_routed_experts, D) <= 200 * 1024

    def _moe_norm_bwd(self, moe, dxs, dst, dsh, dlog, norm):
        """g = dsh + un-permuted dxs + dlog @ W_gate, then the RMSNorm backward of g
        (norm = (x, weight param, rstd, dres fp32 accumulated, dres bf16 copy))."""
        x, nw, rstd, dres, dres_b = norm
        self.C.moe_norm_bwd(dxs, dst, dsh, dlog, self.w(moe.gate.weight), x, self.f32(nw), rstd, dres, dres_b,
                            self.g(nw))

    def _moe_fwd(self, moe, xn, resid_in):
        """Returns (ctx, resid_in + MoE(xn)) as a new fp32 tensor."""
        if self.use_ep:
            return self._moe_fwd_ep(moe, xn, resid_in)
        C = self.C
        T = xn.shape[0]
        E, k, I = moe.n_routed_experts, moe.topk, moe.moe_inter_dim
        idx, wts, ssel, counts, Ep = self._router(moe, xn)
        self._mark("router fwd")
        P = _pad(T * k + E * 255, 256)       # expert ranges are 256-row aligned (CTA-pair tiles)
        row_off = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        tile_group = torch.empty(P // 128, dtype=torch.int32, device=self.device)
        cursor = torch.empty(E, dtype=torch.int32, device=self.device)
        src = torch.empty(P, dtype=torch.int32, device=self.device)
        dst = torch.empty(T, k, dtype=torch.int32, device=self.device)
        C.permute_plan(counts, row_off, tile_group, cursor, src, src_tail_only=True)
        xs = torch.empty(P, self.D, dtype=BF16, device=self.device)
        C.permute_gather(idx, counts, row_off, cursor, xn, src, dst, xs)   # expert-sorted rows in one pass
        self._mark("moe permute fwd")
        w1 = moe.experts[0].w1.weight
        h = torch.empty(P, I, dtype=BF16, device=self.device)
        gu = torch.empty(P, 2 * I, dtype=BF16, device=self.device)
        C.swiglu_fwd(xs, self.swiglu_w13(w1, E), tile_group, h, gu, group_rows=256)
        self._mark("experts gate/up fwd")
        out = torch.empty_like(resid_in) if moe.shared_experts else resid_in.clone()
        shared = []

        def shared_fwd():
            for i, e in enumerate(moe.shared_experts):
                shared.append(self._swiglu_dense_fwd(e.w1.weight, e.w2.weight, xn, out, resid_in if i == 0 else None))
        # the shared experts run on a side stream beside the routed experts'
        # permutation and grouped GEMMs (joined before the combine adds into out)
        side = self._fork(shared_fwd) if moe.shared_experts else None
        ys = torch.empty(P, self.D, dtype=BF16, device=self.device)
        C.grouped_fwd(h, self.stacked(moe.experts[0].w2.weight, E), tile_group, ys, group_rows=256)
        self._mark("experts down fwd")
        self._join(side)
        self._mark("shared experts join")
        C.combine_fwd(ys, dst, wts, out)
        return _Ctx(idx=idx, wts=wts, ssel=ssel, row_off=row_off, tile_group=tile_group, src=src, dst=dst, xs=xs,
                    h=h, gu=gu, ys=ys, shared=shared, Ep=Ep, counts=counts), out

    def _moe_bwd(self, moe, ctx, xn, dres_bf16, dxn_acc, norm=None):
        """MoE backward into dxn_acc (fp32).  With norm = (x, weight, rstd, dres,
        dres_b) and a fusable shape, the FFN norm's backward runs fused with the
        input-gradient sum instead (dxn_acc then holds only the shared experts'
        part) and True is returned."""
        if self.use_ep:
            return self._moe_bwd_ep(moe, ctx, xn, dres_bf16, dxn_acc, norm)
        C = self.C
        T = xn.shape[0]
        E, k, I = moe.n_routed_experts, moe.topk, moe.moe_inter_dim
        fused = self._norm_fusable(moe, norm)
        if not moe.shared_experts and not fused:
            dxn_acc.zero_()

        def shared_bwd():
            for i, (e, sctx) in enumerate(zip(moe.shared_experts, ctx.shared)):
                self._swiglu_dense_bwd(e.w1.weight, e.w2.weight, sctx, xn, dres_bf16, dxn_acc, accumulate=i > 0)
        # shared experts on a side stream beside the routed backward; joined
        # before the un-permute adds the routed input gradients into dxn_acc
        side = self._fork(shared_bwd) if moe.shared_experts else None
        P = ctx.xs.shape[0]
        dys = torch.empty(P, self.D, dtype=BF16, device=self.device)
        dw = torch.empty(T, k, dtype=F32, device=self.device)
        C.combine_bwd(dres_bf16, ctx.ys, ctx.src, ctx.wts, k, dys, dw)
        self._mark("combine bwd")
        w1 = moe.experts[0].w1.weight
        w2 = moe.experts[0].w2.weight
        dgu = torch.empty(P, 2 * I, dtype=BF16, device=self.device)
        C.swiglu_dgrad(dys, self.stacked(w2, E), ctx.tile_group, ctx.gu, dgu, group_rows=256)
        self._mark("experts swiglu dgrad")
        C.grouped_wgrad(dys, ctx.h, ctx.row_off, self.stacked(w2, E, grad=True))
        self._mark("experts down wgrad")
        dxs = torch.empty(P, self.D, dtype=BF16, device=self.device)
        C.grouped_dgrad(dgu, self.swiglu_w13(w1, E).view(E, 2 * I, self.D), ctx.tile_group, dxs, group_rows=256)
        self._mark("experts dgrad")
        C.grouped_wgrad(dgu, ctx.xs, ctx.row_off, self.swiglu_g13(w1, E))
        self._mark("experts up wgrad")
        self._join(side)
        self._mark("shared experts join")
        if fused:
            dlog = self._router_dlog(moe, ctx, xn, dw)
            self._moe_norm_bwd(moe, dxs, ctx.dst, dxn_acc if moe.shared_experts else None, dlog, norm)
            self._mark("router bwd + norm bwd")
            return True
        C.unpermute_bwd(dxs, ctx.dst, dxn_acc)
        self._router_bwd(moe, ctx, xn, dw, dxn_acc)
        self._mark("router bwd")
        return False

    # ------------------------------------------------------------------ MTP
    def _mtp_fwd(self, mod, h_prev, emb, Bm, Sm):
        """One MTP depth on [Bm*Sm] rows: returns (ctx, normalised hidden bf16, pre-norm fp32 hidden)."""
        C, D = self.C, self.D
        blk = mod.block
        T = h_prev.shape[0]
        cat = torch.empty(T, 2 * D, dtype=BF16, device=self.device)
        rh = torch.empty(T, dtype=F32, device=self.device)
        re = torch.empty(T, dtype=F32, device=self.device)
        C.rmsnorm_fwd(h_prev, self.f32(blk.norm_h.weight), 1e-6, cat[:, :D], rh)
        C.rmsnorm_fwd(emb, self.f32(blk.norm_e.weight), 1e-6, cat[:, D:], re)
        f = self._linear(cat, blk.proj.weight, out_dtype=F32)           # fp32 residual of the block
        a_in, ra = self._norm(f, blk.norm_attn.weight)
        qkv = self._linear(a_in, blk.attn.in_proj_weight)               # [T, 3D]
        H = blk.n_heads
        hd = D // H
        Q = torch.empty(Bm * H, Sm, hd, dtype=BF16, device=self.device)
        K = torch.empty_like(Q)
        Vt = torch.empty_like(Q)
        C.heads_pack(qkv, 0, H, hd, Sm, Q)
        C.heads_pack(qkv, D, H, hd, Sm, K)
        C.heads_pack(qkv, 2 * D, H, hd, Sm, Vt)
        O = torch.empty(T, D, dtype=BF16, device=self.device)
        L = torch.empty(Bm * H, Sm, dtype=F32, device=self.device)
        C.flash_fwd(Q, K, Vt, O, L, 0, hd ** -0.5, True, H)
        f2 = torch.empty_like(f)
        C.linear_fwd(O, self.w(blk.attn.out_proj.weight), f2, True, f)
        x_ffn, rf = self._norm(f2, blk.norm_ffn.weight)
        f3 = torch.empty_like(f2)
        ffn = self._swiglu_dense_fwd(blk.w1.weight, blk.w2.weight, x_ffn, f3, f2)
        hn, rn = self._norm(f3, mod.norm.weight)
        ctx = _Ctx(h_prev=h_prev, emb=emb, cat=cat, rh=rh, re=re, f=f, a_in=a_in, ra=ra, qkv=qkv, Q=Q, K=K, V=Vt,
                   O=O, L=L, f2=f2, x_ffn=x_ffn, rf=rf, ffn=ffn, f3=f3, rn=rn, hn=hn, Bm=Bm, Sm=Sm)
        return ctx, hn, f3

    def _mtp_bwd(self, mod, ctx, dhn, dprev_acc, demb):
        """dhn: fp32 grad of the normalised MTP hidden.  Adds d(h_prev) into
        ``dprev_acc`` (fp32) and writes d(emb) (fp32) into ``demb``."""
        C, D = self.C, self.D
        blk = mod.block
        T = ctx.h_prev.shape[0]
        H = blk.n_heads
        hd = D // H
        Bm, Sm = ctx.Bm, ctx.Sm
        df = torch.zeros(T, D, dtype=F32, device=self.device)
        dfb = torch.empty(T, D, dtype=BF16, device=self.device)
        C.rmsnorm_bwd(dhn, ctx.f3, self.f32(mod.norm.weight), ctx.rn, df, None, dfb, self.g(mod.norm.weight))
        dx_ffn = torch.empty(T, D, dtype=F32, device=self.device)
        self._swiglu_dense_bwd(blk.w1.weight, blk.w2.weight, ctx.ffn, ctx.x_ffn, dfb, dx_ffn, accumulate=False)
        C.rmsnorm_bwd(dx_ffn, ctx.f2, self.f32(blk.norm_ffn.weight), ctx.rf, df, None, dfb, self.g(blk.norm_ffn.weight))
        dO = self._linear_bwd(dfb, ctx.O, blk.attn.out_proj.weight)
        dQ = torch.zeros(Bm * H, Sm, hd, dtype=F32, device=self.device)
        dK = torch.empty_like(dQ)
        dV = torch.empty_like(dQ)
        delta = torch.empty(Bm * H, Sm, dtype=F32, device=self.device)
        C.flash_bwd(ctx.Q, ctx.K, ctx.V, ctx.O, dO, ctx.L, delta, dQ, dK, dV, 0, hd ** -0.5, True, H)
        dqkv = torch.empty(T, 3 * D, dtype=BF16, device=self.device)
        C.heads_unpack(dQ, H, hd, Sm, dqkv, 0)
        C.heads_unpack(dK, H, hd, Sm, dqkv, D)
        C.heads_unpack(dV, H, hd, Sm, dqkv, 2 * D)
        da = torch.empty(T, D, dtype=F32, device=self.device)
        self._linear_bwd(dqkv, ctx.a_in, blk.attn.in_proj_weight, dx_acc=da, accumulate=False)
        C.rmsnorm_bwd(da, ctx.f, self.f32(blk.norm_attn.weight), ctx.ra, df, None, dfb, self.g(blk.norm_attn.weight))
        dcat = self._linear_bwd(dfb, ctx.cat, blk.proj.weight)
        C.rmsnorm_bwd(dcat[:, :D], ctx.h_prev, self.f32(blk.norm_h.weight), ctx.rh, dprev_acc, None, None,
                      self.g(blk.norm_h.weight))
        C.rmsnorm_bwd(dcat[:, D:], ctx.emb, self.f32(blk.norm_e.weight), ctx.re, demb, None, None,
                      self.g(blk.norm_e.weight))

    # ------------------------------------------------------------ full step
    def _layer_fwd(self, layer, x, B, S):
        """One transformer block on the fp32 residual ``x``: returns (saved tensors, next residual)."""
        C = self.C
        xn1, r1 = self._norm(x, layer.attn_norm.weight)
        actx = self._mla_fwd(layer.attn, xn1, B, S)
        x_mid = torch.empty_like(x)
        C.linear_fwd(actx.O, self.w(layer.attn.wo.weight), x_mid, True, x)
        xn2, r2 = self._norm(x_mid, layer.ffn_norm.weight)
        self._mark("o-proj fwd")
        if hasattr(layer.ffn, "experts"):
            fctx, x_next = self._moe_fwd(layer.ffn, xn2, x_mid)
            self._mark("moe fwd")
        else:
            x_next = torch.empty_like(x_mid)
            fctx = self._swiglu_dense_fwd(layer.ffn.w1.weight, layer.ffn.w2.weight, xn2, x_next, x_mid)
            self._mark("dense ffn fwd")
        return (x, r1, actx, x_mid, xn2, r2, fctx), x_next

    @property
    def _empty_i32(self):
        if not hasattr(self, "_e_i32"):
            self._e_i32 = torch.empty(0, dtype=torch.int32, device=self.device)
        return self._e_i32

    def forward_backward(self, tokens: torch.Tensor, targets: torch.Tensor, loss_scale: float = 1.0) -> Dict:
        """One micro-batch: forward, loss, backward (gradients accumulate).

        Returns device tensors ``loss`` (main CE), ``mtp_loss`` (or None) and
        ``balance_loss``; nothing here synchronises with the host.  With
        ``use_graphs`` the whole micro-step is captured once per input shape
        into a CUDA graph and replayed (no per-kernel host launch cost).
        """
        if self.use_graphs and torch.cuda.is_current_stream_capturing() is False:
            return self._graphed(tokens, targets, loss_scale)
        return self._forward_backward(tokens, targets, loss_scale)

    def _graphed(self, tokens, targets, loss_scale):
        timer = self.phase_timer
        if timer is not None:
            timer.book(timer.take())       # marks issued before this micro-step (host side)
        key = (tuple(tokens.shape), float(loss_scale), timer is not None)
        entry = self._graphs.get(key)
        if entry is None:
            st_tok = tokens.detach().clone()
            st_tgt = targets.detach().clone()
            # The warm-up run really executes: keep the gradients it adds out.
            saved = [f.grad.clone() for f in self.flats]
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._forward_backward(st_tok, st_tgt, loss_scale)
            torch.cuda.current_stream().wait_stream(side)
            if timer is not None:
                timer.take()               # the eager warm-up's marks are not booked
            graph = torch.cuda.CUDAGraph()
            # thread-local capture: a CUDA call from another thread (the data
            # loader's pin-memory thread allocating pinned buffers) must not
            # invalidate this capture
            with _ext.launch_scope() as scope, torch.cuda.graph(graph, capture_error_mode="thread_local"):
                out = self._forward_backward(st_tok, st_tgt, loss_scale)
            marks = timer.take() if timer is not None else None
            for f, g in zip(self.flats, saved):
                f.grad.copy_(g)
            del saved
            entry = (graph, st_tok, st_tgt, out, self._finite, scope.count, marks)
            self._graphs[key] = entry
        graph, st_tok, st_tgt, out, finite, n_kernels, marks = entry
        st_tok.copy_(tokens)
        st_tgt.copy_(targets)
        graph.replay()
        _ext.add_launches(n_kernels)
        if timer is not None:
            timer.book(marks)              # this replay's event-record nodes
        self._finite = finite
        res = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in out.items()}
        self._last_losses = res["loss"]
        return res

    def _range(self, name: Optional[str]) -> None:
        """Open (name) or close (None) an NVTX range when DSV3_NVTX=1."""
        if self.nvtx:
            if name is None:
                torch.cuda.nvtx.range_pop()
            else:
                torch.cuda.nvtx.range_push(name)

    def _seg_tensors(self, seg, segw):
        key = (tuple(seg), tuple(segw))
        got = self._segcache.get(key)
        if got is None:
            got = (torch.tensor(seg, dtype=torch.int32, device=self.device),
                   torch.tensor(segw, dtype=F32, device=self.device))
            self._segcache[key] = got
        return got

    def _forward_backward(self, tokens: torch.Tensor, targets: torch.Tensor, loss_scale: float = 1.0) -> Dict:
        C, m, D = self.C, self.model, self.D
        B, S = tokens.shape
        T = B * S
        tok = tokens.reshape(-1).long().contiguous()
        tgt = targets.reshape(-1).long().contiguous()
        self._mark("between micro-steps")
        x = torch.empty(T, D, dtype=F32, device=self.device)
        C.embedding_fwd(tok, self.f32(m.embed.weight), x)
        self._mark("embedding fwd")
        saved = []
        for li, layer in enumerate(m.layers):
            self._range(f"fwd layer {li}")
            ctx, x_next = self._layer_fwd(layer, x, B, S)
            # with recomputation only the layer input survives the forward pass
            saved.append(x if self.recompute else ctx)
            x = x_next
            self._range(None)
        hL = x
        xf, rf = self._norm(hL, m.norm.weight)

        # MTP depths (h_prev = pre-final-norm hidden, emb = embed(tokens[:, d+1:]))
        mtp_ctx = []
        rows = [xf]
        tgts = [tgt]
        seg = [0, T]
        if self.mtp is not None:
            prev = hL.view(B, S, D)
            for d, mod in enumerate(self.mtp.mtp_modules):
                Sm = S - d - 2
                if Sm <= 0:
                    break
                h_prev = prev[:, :Sm].reshape(B * Sm, D).contiguous()
                etok = tokens[:, d + 1:d + 1 + Sm].reshape(-1).long().contiguous()
                emb = torch.empty(B * Sm, D, dtype=F32, device=self.device)
                C.embedding_fwd(etok, self.f32(m.embed.weight), emb)
                ctx, hn, f3 = self._mtp_fwd(mod, h_prev, emb, B, Sm)
                ctx.etok = etok
                mtp_ctx.append(ctx)
                rows.append(hn)
                tgts.append(tokens[:, d + 2:d + 2 + Sm].reshape(-1).long().contiguous())
                seg.append(seg[-1] + B * Sm)
                prev = hn.float().view(B, Sm, D)  # next depth chains on the normalised hidden
        self._mark("mtp fwd")
        allx = torch.cat(rows, 0) if len(rows) > 1 else xf
        allt = torch.cat(tgts, 0) if len(tgts) > 1 else tgt
        Tt = allx.shape[0]

        # fused LM head + cross-entropy over every row
        head_w = self.w(m.head.weight)
        nt = (self.V + 255) // 256
        pmax = torch.empty(Tt, 2 * nt, dtype=F32, device=self.device)   # one partial per 128-column half tile
        psum = torch.empty(Tt, 2 * nt, dtype=F32, device=self.device)
        tl = torch.zeros(Tt, dtype=F32, device=self.device)
        C.ce_fwd_partials(allx, head_w, allt, pmax, psum, tl)
        lse = torch.empty(Tt, dtype=F32, device=self.device)
        lrows = torch.empty(Tt, dtype=F32, device=self.device)
        C.ce_rows(pmax, psum, tl, allt, lse, lrows)
        nseg = len(seg) - 1
        segw = [1.0] + [self.mtp.mtp_weight / max(1, nseg - 1)] * (nseg - 1) if self.mtp is not None else [1.0]
        seg_t, segw_t = self._seg_tensors(seg, segw)
        losses = torch.empty(nseg, dtype=F32, device=self.device)
        rscale = torch.empty(Tt, dtype=F32, device=self.device)
        C.ce_reduce(lrows, allt, seg_t, segw_t, float(loss_scale), losses, rscale)
        self._last_losses = losses

        self._mark("ce fwd")
        # ---------------- backward
        dall = torch.empty(Tt, D, dtype=F32, device=self.device)
        dlog = torch.empty(min(self.ce_chunk, Tt), self.Vp, dtype=BF16, device=self.device)
        for a in range(0, Tt, self.ce_chunk):
            b = min(Tt, a + self.ce_chunk)
            dl = dlog[:b - a]
            C.ce_bwd_logits(allx[a:b], head_w, allt[a:b], lse[a:b], rscale[a:b], dl)
            C.linear_wgrad(dl[:, :self.V], allx[a:b], self.g(m.head.weight))
            C.linear_dgrad(dl[:, :self.V], head_w, dall[a:b], False)
        del dlog
        self._mark("ce bwd")
        dres = torch.zeros(T, D, dtype=F32, device=self.device)
        if mtp_ctx:
            # Depth d+1 consumed the first rows of depth d's normalised hidden,
            # so its input gradient is carried back into depth d's output grad.
            carry, carry_rows = None, 0
            for d in range(len(mtp_ctx) - 1, -1, -1):
                ctx = mtp_ctx[d]
                mod = self.mtp.mtp_modules[d]
                dhn = dall[seg[d + 1]:seg[d + 2]]
                if carry is not None:
                    dhn = dhn.clone()
                    dhn.view(B, ctx.Sm, D)[:, :carry_rows].add_(carry.view(B, carry_rows, D))
                dprev = torch.zeros(ctx.h_prev.shape, dtype=F32, device=self.device)
                demb = torch.zeros(ctx.emb.shape, dtype=F32, device=self.device)
                self._mtp_bwd(mod, ctx, dhn.contiguous(), dprev, demb)
                C.embedding_bwd(ctx.etok, demb, self.g(m.embed.weight))
                if d == 0:
                    dres.view(B, S, D)[:, :ctx.Sm].add_(dprev.view(B, ctx.Sm, D))
                else:
                    carry, carry_rows = dprev, ctx.Sm
        self._mark("mtp bwd")
        dres_b = torch.empty(T, D, dtype=BF16, device=self.device)
        C.rmsnorm_bwd(dall[:T], hL, self.f32(m.norm.weight), rf, dres, None, dres_b, self.g(m.norm.weight))
        for li, (layer, kept) in enumerate(zip(reversed(m.layers), reversed(saved))):
            self._range(f"bwd layer {len(saved) - 1 - li}")
            if self.recompute:
                kept, _ = self._layer_fwd(layer, kept, B, S)
                self._mark("recompute fwd")
            x_in, r1, actx, x_mid, xn2, r2, fctx = kept
            dxn2 = torch.empty(T, D, dtype=F32, device=self.device)
            normed = False
            if hasattr(layer.ffn, "experts"):
                normed = self._moe_bwd(layer.ffn, fctx, xn2, dres_b, dxn2,
                                       norm=(x_mid, layer.ffn_norm.weight, r2, dres, dres_b))
                self._mark("moe bwd")
            else:
                self._swiglu_dense_bwd(layer.ffn.w1.weight, layer.ffn.w2.weight, fctx, xn2, dres_b, dxn2,
                                       accumulate=False)
                self._mark("dense ffn bwd")
            if not normed:
                C.rmsnorm_bwd(dxn2, x_mid, self.f32(layer.ffn_norm.weight), r2, dres, None, dres_b,
                              self.g(layer.ffn_norm.weight))
            dxn1 = torch.empty(T, D, dtype=F32, device=self.device)
            self._mla_bwd(layer.attn, actx, dres_b, dxn1, B, S)
            C.rmsnorm_bwd(dxn1, x_in, self.f32(layer.attn_norm.weight), r1, dres, None, dres_b,
                          self.g(layer.attn_norm.weight))
            self._range(None)
        C.embedding_bwd(tok, dres, self.g(m.embed.weight))
        self._mark("embedding bwd")

        balance = torch.zeros((), device=self.device)
        out = {"loss": losses[0], "mtp_loss": losses[1:].mean() if nseg > 1 else None, "balance_loss": balance}
        self._finite = torch.isfinite(losses).all()
        return out

    # ------------------------------------------------------------ optimizer
    def last_loss_finite(self) -> bool:
        """Whether the last micro-batch's losses are finite on *every* rank
        (ranks must agree, or they would take different collective paths)."""
        if self.dp is not None:
            flag = self._finite.to(torch.int32).reshape(1)
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN, group=self.dp.group)
            return bool(flag.item())
        return bool(self._finite)

    def clip_and_step(self, max_norm: float) -> None:
        self._mark("between micro-steps")
        if self.dp is not None and hasattr(self.dp, "step"):
            # optimizer.step() runs the reduce-scatter + sharded AdamW + all-gather
            self.dp.max_norm = float(max_norm)
            self.optimizer.step()
        else:
            if self.dp is not None:
                self.dp.reduce_gradients()
            extra = self.dp.extra_sqsum() if self.dp is not None else None
            self.optimizer.compute_clip(max_norm, extra)
            self.optimizer.step()
            if self.dp is not None:
                self.dp.after_step()
        self._mark("optimizer step" if self.dp is None else "data-parallel optimizer step")

    def zero_grad(self) -> None:
        self.optimizer.zero_grad()

    def check(self) -> None:
        check_status()

    def close(self) -> None:
        """Release captured graphs and the expert-parallel peer mappings
        (before the process group goes away)."""
        torch.cuda.synchronize(self.device)
        self._graphs.clear()
        if self.ep is not None:
            self.ep.close()
            self.ep = None
        if self.dp_heap is not None:
            # the module parameters alias the heap: move them to plain memory first
            for f in self.flats:
                for name in ("master", "grad", "shadow"):
                    setattr(f, name, getattr(f, name).clone())
                f.rebind()
            self.optimizer._bind_state()
            self.dp_heap.close()
            self.dp_heap = None

    # ---------------------------------------------------- module interplay
    def sync_to_modules(self) -> None:
        """Module parameters already alias the flat masters; re-point any that
        were replaced (e.g. by ``load_state_dict``)."""
        for f in self.flats:
            f.pull_from_params()

    def sync_from_modules(self) -> None:
        for f in self.flats:
            f.pull_from_params()
        self.optimizer._bind_state()

    def expert_shard_state(self) -> Dict[str, torch.Tensor]:
        """This rank's routed experts (sharded training): fp32 weights under
        their state-dict names and AdamW moments under ``exp_avg.`` /
        ``exp_avg_sq.`` prefixes, as views into the flat buffers."""
        f, opt = self.flat_expert, self.optimizer
        fi = self.flats.index(f)
        out: Dict[str, torch.Tensor] = {}
        for n, p in self._local_expert_named:
            out[n] = f.view(f.master, p)
            out["exp_avg." + n] = f.view(opt.exp_avg[fi], p)
            out["exp_avg_sq." + n] = f.view(opt.exp_avg_sq[fi], p)
        return out

    def load_expert_shard_state(self, tensors: Dict[str, torch.Tensor]) -> None:
        """Inverse of ``expert_shard_state`` (the shard must cover exactly
        this rank's experts)."""
        mine = self.expert_shard_state()
        missing = [k for k in mine if k not in tensors]
        extra = [k for k in tensors if k not in mine]
        if missing or extra:
            raise RuntimeError(f"expert shard does not match this rank's experts: {len(missing)} missing "
                               f"({missing[:3]}), {len(extra)} unexpected ({extra[:3]})")
        for k, dst in mine.items():
            dst.copy_(tensors[k].reshape(dst.shape))
        self.flat_expert.refresh_shadow()

    def optimizer_state_for_checkpoint(self) -> dict:
        """torch-AdamW state dict with standalone tensors (reference layout)."""
        full = None
        if self.dp is not None and hasattr(self.dp, "gather_moments"):
            full = self.dp.gather_moments(self.optimizer)   # collective: every rank calls it
            self.optimizer._bind_state(full)
        try:
            sd = self.optimizer.state_dict()
            for st in sd["state"].values():
                for k in ("exp_avg", "exp_avg_sq"):
                    if k in st:
                        st[k] = st[k].clone()
                if "step" in st:
                    st["step"] = st["step"].clone()
        finally:
            if full is not None:
                self.optimizer._bind_state()
        return sd
