"""Flat parameter storage and the fused AdamW optimizer.

``FlatParams`` moves a list of parameters into one contiguous fp32 master
buffer and re-points every ``Parameter.data`` (and ``.grad``) at a view of
it, so the module tree, ``state_dict`` keys and optimizer parameter order of
the reference are untouched while the kernels see large contiguous buffers:

* ``master`` fp32 - the weights the optimizer updates (checkpoints are fp32);
* ``grad`` fp32 - weight-gradient GEMMs accumulate into it in place, across
  micro-batches, so gradient accumulation costs nothing extra;
* ``shadow`` bf16 - what the GEMMs read; refreshed by the AdamW kernel.

Parameters are laid out in *blocks*: the parameters of a block are adjacent
with no padding (e.g. ``[w1_e0, w3_e0, w1_e1, w3_e1, ...]`` forms the
``[E, 2, I, D]`` operand of the grouped SwiGLU GEMM); blocks start on
64-element boundaries (TMA needs 16-byte aligned bases).

``FlatAdamW`` is a ``torch.optim.Optimizer`` (so ``LambdaLR`` drives its
``lr``) whose ``step`` runs the fused kernels over the flat buffers.  Its
``state_dict`` is the torch AdamW layout (``step``, ``exp_avg``,
``exp_avg_sq`` per parameter, same parameter indices), so optimizer files are
interchangeable with the reference's.  Under the peer-memory data-parallel
step a flat's moments can be sharded (``shard_moments``): the rank keeps only
its own range and the full moments exist only while a checkpoint is written.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from ._ext import native

ALIGN = 64


class FlatParams:
    """One fp32 master / fp32 grad / bf16 shadow buffer over blocks of parameters."""

    @staticmethod
    def layout_numel(blocks: Sequence[Sequence[torch.nn.Parameter]]) -> int:
        """Elements of the buffers ``FlatParams(blocks)`` allocates."""
        off = 0
        for block in blocks:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            off += sum(p.numel() for p in block)
        return (off + ALIGN - 1) // ALIGN * ALIGN

    def __init__(self, blocks: Sequence[Sequence[torch.nn.Parameter]], device, alloc=None):
        """``alloc(name, numel, dtype)`` may supply the three buffers (zeroed),
        e.g. from a symmetric heap; by default they are plain device tensors."""
        self.params: List[torch.nn.Parameter] = []
        self.offsets: Dict[int, int] = {}
        self.block_offsets: List[int] = []
        off = 0
        for block in blocks:
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            self.block_offsets.append(off)
            for p in block:
                if id(p) in self.offsets:
                    raise ValueError("parameter listed twice in FlatParams")
                self.offsets[id(p)] = off
                self.params.append(p)
                off += p.numel()
        self.numel = (off + ALIGN - 1) // ALIGN * ALIGN
        if alloc is None:
            def alloc(name, n, dtype):
                return torch.zeros(n, dtype=dtype, device=device)
        self.master = alloc("master", self.numel, torch.float32)
        self.grad = alloc("grad", self.numel, torch.float32)
        self.shadow = alloc("shadow", self.numel, torch.bfloat16)
        for p in self.params:
            o = self.offsets[id(p)]
            self.master[o:o + p.numel()].copy_(p.data.reshape(-1).to(device=device, dtype=torch.float32))
        self.rebind()
        self.refresh_shadow()

    def view(self, buf: torch.Tensor, p: torch.nn.Parameter) -> torch.Tensor:
        o = self.offsets[id(p)]
        return buf[o:o + p.numel()].view(p.shape)

    def block_view(self, buf: torch.Tensor, first: torch.nn.Parameter, shape) -> torch.Tensor:
        """View of ``buf`` starting at ``first`` with ``shape`` (spans a whole block)."""
        o = self.offsets[id(first)]
        n = 1
        for s in shape:
            n *= s
        return buf[o:o + n].view(*shape)

    def rebind(self) -> None:
        """Point every parameter (and its grad) back at the flat buffers."""
        for p in self.params:
            p.data = self.view(self.master, p)
            p.grad = self.view(self.grad, p)

    def pull_from_params(self) -> None:
        """Copy parameter values into the master buffer if something replaced
        ``Parameter.data`` (e.g. ``load_state_dict``), then rebind."""
        for p in self.params:
            v = self.view(self.master, p)
            if p.data.data_ptr() != v.data_ptr():
                v.copy_(p.data.reshape(v.shape))
        self.rebind()
        self.refresh_shadow()

    def refresh_shadow(self) -> None:
        native().cast_f32_bf16(self.master, self.shadow)

    def zero_grad(self) -> None:
        self.grad.zero_()
        for p in self.params:
            if p.grad is None or p.grad.data_ptr() != self.view(self.grad, p).data_ptr():
                p.grad = self.view(self.grad, p)


class FlatAdamW(torch.optim.Optimizer):
    """AdamW (torch semantics) over ``FlatParams`` buffers with fused kernels.

    ``param_groups`` are the reference's two groups (decayed params with
    ``dim >= 2``, the rest undecayed) in the reference's order.  ``flats``
    hold the parameters; ``flat_groups[i]`` is the param group whose
    hyperparameters apply to ``flats[i]`` (default: flat i <-> group i).  A
    parameter held by no flat (a routed expert owned by another rank when
    experts are sharded) has no optimizer state here.
    """

    def __init__(self, groups, flats: Sequence[FlatParams], lr: float, betas=(0.9, 0.95), eps: float = 1e-8,
                 flat_groups: Optional[Sequence[int]] = None):
        super().__init__(groups, dict(lr=lr, betas=betas, eps=eps, weight_decay=0.0, amsgrad=False,
                                      maximize=False, foreach=None, capturable=False, differentiable=False,
                                      fused=None))
        self.flats = list(flats)
        if flat_groups is None:
            if len(self.flats) != len(self.param_groups):
                raise ValueError("one FlatParams per param group unless flat_groups is given")
            flat_groups = list(range(len(self.flats)))
        self.flat_groups = list(flat_groups)
        self._flat_of = {}
        for fi, f in enumerate(self.flats):
            for p in f.params:
                self._flat_of[id(p)] = fi
        dev = self.flats[0].master.device
        self.exp_avg = [torch.zeros_like(f.master) for f in self.flats]
        self.exp_avg_sq = [torch.zeros_like(f.master) for f in self.flats]
        self.step_count = 0
        # flat index -> (lo, hi): the moments of that flat hold only [lo, hi)
        self.moment_range: Dict[int, tuple] = {}
        # replaces the local update when set (the data-parallel step); called
        # from ``step`` so the LR scheduler sees a regular optimizer step
        self.stepper = None
        self._scratch = torch.empty(1024 * 4, device=dev)
        self.sqsum = torch.zeros(1, device=dev)
        self.grad_norm = torch.zeros(1, device=dev)
        self.clip = torch.ones(1, device=dev)
        self._bind_state()

    def shard_moments(self, fi: int, lo: int, hi: int) -> None:
        """Keep only elements ``[lo, hi)`` of flat ``fi``'s AdamW moments (this rank's shard)."""
        self.exp_avg[fi] = self.exp_avg[fi][lo:hi].clone()
        self.exp_avg_sq[fi] = self.exp_avg_sq[fi][lo:hi].clone()
        self.moment_range[fi] = (lo, hi)
        self._bind_state()

    def _bind_state(self, full: Optional[Dict[int, tuple]] = None) -> None:
        """Point ``state[p]`` at views of the moment buffers.  A sharded flat
        binds only ``step`` unless ``full`` supplies its gathered
        ``(exp_avg, exp_avg_sq)`` full-size buffers (checkpoint writing)."""
        for group in self.param_groups:
            for p in group["params"]:
                fi = self._flat_of.get(id(p))
                if fi is None:
                    self.state.pop(p, None)
                    continue
                f = self.flats[fi]
                st = {"step": torch.tensor(float(self.step_count))}
                if fi not in self.moment_range:
                    st.update(exp_avg=f.view(self.exp_avg[fi], p), exp_avg_sq=f.view(self.exp_avg_sq[fi], p))
                elif full is not None and fi in full:
                    st.update(exp_avg=f.view(full[fi][0], p), exp_avg_sq=f.view(full[fi][1], p))
                self.state[p] = st

    def compute_clip(self, max_norm: float, extra_sqsum: Optional[torch.Tensor] = None) -> None:
        """Global grad norm over all flats (plus ``extra_sqsum`` from other
        ranks / shards) and the clip coefficient, on the device."""
        C = native()
        C.grad_sqsum([f.grad for f in self.flats], self._scratch, self.sqsum)
        if extra_sqsum is not None:
            self.sqsum.add_(extra_sqsum)
        C.clip_coef(self.sqsum, float(max_norm), self.grad_norm, self.clip)

    def step_flat(self, fi: int, coef: Optional[torch.Tensor] = None) -> None:
        """AdamW over flat ``fi`` (the step counter must already be advanced)."""
        C = native()
        f = self.flats[fi]
        group = self.param_groups[self.flat_groups[fi]]
        b1, b2 = group["betas"]
        n_decay = f.numel if group["weight_decay"] > 0 else 0
        C.adamw_flat(f.master, f.grad, self.exp_avg[fi], self.exp_avg_sq[fi], f.shadow, n_decay,
                     float(group["lr"]), float(b1), float(b2), float(group["eps"]),
                     float(group["weight_decay"]), self.step_count, self.clip if coef is None else coef)

    def mark_step(self) -> None:
        """Advance the per-parameter ``step`` entries to ``step_count``."""
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st is not None:
                    st["step"].fill_(float(self.step_count))

    @torch.no_grad()
    def step(self, closure=None):
        if self.stepper is not None:
            self.stepper(self)
            return None
        self.step_count += 1
        for fi in range(len(self.flats)):
            self.step_flat(fi)
        self.mark_step()
        return None

    def zero_grad(self, set_to_none: bool = True) -> None:
        for f in self.flats:
            f.zero_grad()

    def load_state_dict(self, state_dict) -> None:
        """Load a torch-AdamW state dict, copying moments into the flat buffers."""
        super().load_state_dict(state_dict)
        steps = []
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p, {})
                fi = self._flat_of.get(id(p))
                if "exp_avg" in st and fi is not None:
                    f = self.flats[fi]
                    if fi in self.moment_range:
                        # copy only the part of p inside this rank's shard
                        lo, hi = self.moment_range[fi]
                        o = f.offsets[id(p)]
                        a, b = max(lo, o), min(hi, o + p.numel())
                        if a < b:
                            for dst, key in ((self.exp_avg[fi], "exp_avg"), (self.exp_avg_sq[fi], "exp_avg_sq")):
                                dst[a - lo:b - lo].copy_(st[key].reshape(-1)[a - o:b - o])
                    else:
                        f.view(self.exp_avg[fi], p).copy_(st["exp_avg"].reshape(p.shape))
                        f.view(self.exp_avg_sq[fi], p).copy_(st["exp_avg_sq"].reshape(p.shape))
                    steps.append(int(float(st["step"])))
        if steps:
            self.step_count = max(steps)
        self._bind_state()
