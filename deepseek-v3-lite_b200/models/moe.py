"""DeepSeekMoE: sigmoid top-k routing, shared experts, aux-loss-free balancing.

Semantics (reference ``models/moe.py:7-201``):

* gate: ``s = sigmoid(x W^T)``; experts are *selected* on ``s + bias`` (the
  bias is an fp32 buffer, never a parameter, and gets no gradient), while the
  mixing weights come from the *unbiased* scores, normalised to sum to one and
  multiplied by ``route_scale``;
* output ``sum_k w_k * expert_k(x) + sum_s shared_s(x)`` (no 1/n on shared);
* bias update from the last forward's per-expert counts: over
  ``mean * (1 + upper)`` -> ``bias -= speed``; under ``mean * (1 - lower)`` ->
  ``bias += speed``;
* diagnostic balance metric ``E * sum_e f_e * P_e``.

The routed computation is the hot path.  On CUDA it runs as: fused router
kernel -> expert-sorted, tile-padded permutation -> tcgen05 grouped GEMM with
a SwiGLU epilogue -> grouped down-projection -> weighted combine
(``ops.moe``).  There is no host synchronisation and no per-expert Python
loop.  On CPU the per-expert loop below is the numerics oracle.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class AuxLossFreeGate(nn.Module):
    """Sigmoid top-k router with a selection-only bias."""

    def __init__(self, config: dict):
        super().__init__()
        self.dim = config["dim"]
        self.topk = config["n_activated_experts"]
        self.n_routed_experts = config["n_routed_experts"]
        self.route_scale = config.get("route_scale", 1.0)
        self.bias_upper = config.get("bias_upper_threshold", 0.10)
        self.bias_lower = config.get("bias_lower_threshold", 0.10)
        self.weight = nn.Parameter(torch.empty(self.n_routed_experts, self.dim))
        nn.init.normal_(self.weight, std=0.006)
        self.register_buffer("bias", torch.zeros(self.n_routed_experts, dtype=torch.float32))

    @torch.no_grad()
    def update_bias(self, counts: torch.Tensor, speed: float = 0.001) -> None:
        """Move the selection bias away from over-/under-loaded experts (deadband)."""
        counts = counts.to(torch.float32).to(self.bias.device)
        mean = counts.mean()
        over = counts > mean * (1.0 + self.bias_upper)
        under = counts < mean * (1.0 - self.bias_lower)
        self.bias.sub_(over.to(self.bias.dtype) * speed)
        self.bias.add_(under.to(self.bias.dtype) * speed)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Return ``(weights [T, k], indices [T, k])`` for flat tokens ``x [T, dim]``."""
        scores = torch.sigmoid(F.linear(x, self.weight))
        chosen = torch.topk(scores + self.bias.to(scores.dtype), self.topk, dim=-1).indices
        picked = scores.gather(1, chosen)
        norm = picked.sum(dim=-1, keepdim=True).clamp(min=1e-10)
        return (picked / norm * self.route_scale).to(x.dtype), chosen


class Expert(nn.Module):
    """SwiGLU expert ``w2(silu(w1 x) * w3 x)``."""

    def __init__(self, dim: int, inter_dim: int):
        super().__init__()
        self.w1 = nn.Linear(dim, inter_dim, bias=False)
        self.w2 = nn.Linear(inter_dim, dim, bias=False)
        self.w3 = nn.Linear(dim, inter_dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class DeepSeekMoE(nn.Module):
    """Routed + shared SwiGLU experts with aux-loss-free bias balancing."""

    def __init__(self, config: dict):
        super().__init__()
        self.dim = config["dim"]
        self.n_routed_experts = config["n_routed_experts"]
        self.n_shared_experts = config["n_shared_experts"]
        self.moe_inter_dim = config["moe_inter_dim"]
        self.topk = config["n_activated_experts"]
        # the configured value, as the reference keeps it; every accepted value
        # runs the same native grouped kernels on CUDA and the same PyTorch
        # math on the CPU
        self.moe_dispatch = config.get("moe_dispatch", "stacked")
        self.gate = AuxLossFreeGate(config)
        self.experts = nn.ModuleList(Expert(self.dim, self.moe_inter_dim) for _ in range(self.n_routed_experts))
        self.shared_experts = nn.ModuleList(Expert(self.dim, self.moe_inter_dim) for _ in range(self.n_shared_experts))
        self._last_weights: Optional[torch.Tensor] = None
        self._last_indices: Optional[torch.Tensor] = None
        # Per-expert token counts of the last forward (device tensor, no sync).
        self._last_counts: Optional[torch.Tensor] = None

    # Stacked views of the live expert weights, rebuilt on every access so they
    # can never go stale after an optimizer step.
    @property
    def _stacked_w1(self) -> torch.Tensor:
        return torch.stack([e.w1.weight for e in self.experts])

    @property
    def _stacked_w2(self) -> torch.Tensor:
        return torch.stack([e.w2.weight for e in self.experts])

    @property
    def _stacked_w3(self) -> torch.Tensor:
        return torch.stack([e.w3.weight for e in self.experts])

    @property
    def _shared_w1(self) -> Optional[torch.Tensor]:
        return torch.stack([e.w1.weight for e in self.shared_experts]) if self.n_shared_experts else None

    @property
    def _shared_w2(self) -> Optional[torch.Tensor]:
        return torch.stack([e.w2.weight for e in self.shared_experts]) if self.n_shared_experts else None

    @property
    def _shared_w3(self) -> Optional[torch.Tensor]:
        return torch.stack([e.w3.weight for e in self.shared_experts]) if self.n_shared_experts else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Route ``x`` (``[..., dim]``) through routed and shared experts."""
        shape = x.shape
        flat = x.reshape(-1, self.dim)
        weights, indices = self.gate(flat)
        self._last_weights = weights.detach()
        self._last_indices = indices.detach()
        self._last_counts = None
        out = self._routed_loop(flat, weights, indices)
        for ex in self.shared_experts:
            out = out + ex(flat)
        return out.view(shape)

    def _routed_loop(self, flat: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """Per-expert gather -> SwiGLU -> weighted scatter-add (CPU oracle)."""
        out = torch.zeros_like(flat)
        token_of = torch.arange(flat.size(0), device=flat.device).unsqueeze(1).expand_as(indices)
        for e, ex in enumerate(self.experts):
            hit = indices == e
            if not bool(hit.any()):
                continue
            rows = token_of[hit]
            y = ex(flat[rows]) * weights[hit].unsqueeze(-1).to(flat.dtype)
            out = out.index_add(0, rows, y.to(out.dtype))
        return out

    def expert_counts(self) -> Optional[torch.Tensor]:
        """Tokens routed to each expert by the last forward (device tensor)."""
        if self._last_counts is not None:
            return self._last_counts
        if self._last_indices is None:
            return None
        return torch.bincount(self._last_indices.flatten(), minlength=self.n_routed_experts)

    def get_load_balance_loss(self) -> torch.Tensor:
        """Diagnostic ``E * sum_e f_e * P_e`` from the last forward (0 before any)."""
        if self._last_weights is None or self._last_indices is None:
            return torch.tensor(0.0, device=self.gate.weight.device)
        idx = self._last_indices.flatten()
        E = self.n_routed_experts
        T = self._last_weights.size(0)
        counts = torch.bincount(idx, minlength=E).float()
        frac = counts / counts.sum().clamp(min=1e-10)
        mass = torch.zeros(E, device=idx.device, dtype=torch.float32)
        mass.index_add_(0, idx, self._last_weights.flatten().float())
        return (frac * (mass / T)).sum() * E

    def update_gate_bias(self, speed: float = 0.001) -> None:
        """Apply the bias rule with the counts of the last forward."""
        counts = self.expert_counts()
        if counts is None:
            return
        self.gate.update_bias(counts, speed=speed)
