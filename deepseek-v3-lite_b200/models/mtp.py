"""Multi-token prediction (MTP) heads.

Semantics (reference ``models/mtp.py:7-120``):

* ``MTPBlock``: ``h = proj([norm_h(prev_h) | norm_e(emb)])``, then a pre-norm
  *standard* multi-head self-attention (bias-free, causal) and a pre-norm
  SwiGLU FFN of width ``inter_dim``, both residual;
* ``MTPModule``: block -> RMSNorm -> the main model's (shared) output head;
* ``MultiTokenPrediction``: depth ``d`` consumes ``h[:, :S-d-2]`` (pre-final-norm
  hidden of the main model for depth 0, the previous MTP hidden after) and
  ``embed(tokens[:, d+1 : d+1+usable])`` and predicts ``tokens[:, d+2 :]``;
  loss = ``CE(main) + w * mean_d CE(mtp_d)`` with ``ignore_index=-100``.

The attention module keeps ``nn.MultiheadAttention``'s parameter names
(``attn.in_proj_weight``, ``attn.out_proj.weight``) so checkpoints interchange
with the reference.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ops import norm as norm_ops


class MTPBlock(nn.Module):
    """Fuse the previous hidden state with the next token's embedding, then refine."""

    def __init__(self, config: dict):
        super().__init__()
        self.dim = config["dim"]
        self.n_heads = config["n_heads"]
        inter = config["inter_dim"]
        self.norm_h = nn.RMSNorm(self.dim, eps=1e-6)
        self.norm_e = nn.RMSNorm(self.dim, eps=1e-6)
        self.proj = nn.Linear(2 * self.dim, self.dim, bias=False)
        self.norm_attn = nn.RMSNorm(self.dim, eps=1e-6)
        self.attn = nn.MultiheadAttention(self.dim, self.n_heads, batch_first=True, bias=False)
        self.norm_ffn = nn.RMSNorm(self.dim, eps=1e-6)
        self.w1 = nn.Linear(self.dim, inter, bias=False)
        self.w2 = nn.Linear(inter, self.dim, bias=False)
        self.w3 = nn.Linear(self.dim, inter, bias=False)
        self._causal_mask_size = 0
        self.register_buffer("_causal_mask", torch.empty(0, 0), persistent=False)

    def _get_causal_mask(self, seqlen: int, device) -> torch.Tensor:
        if seqlen > self._causal_mask_size or self._causal_mask.device != torch.device(device):
            self._causal_mask = torch.full((seqlen, seqlen), float("-inf"), device=device).triu(1)
            self._causal_mask_size = seqlen
        return self._causal_mask[:seqlen, :seqlen]

    def forward(self, prev_hidden: torch.Tensor, target_emb: torch.Tensor) -> torch.Tensor:
        rn = norm_ops.rms_norm
        fused = self.proj(torch.cat([rn(prev_hidden, self.norm_h.weight, self.norm_h.eps),
                                     rn(target_emb, self.norm_e.weight, self.norm_e.eps)], dim=-1))
        a_in = rn(fused, self.norm_attn.weight, self.norm_attn.eps)
        mask = self._get_causal_mask(fused.size(1), fused.device)
        a_out, _ = self.attn(a_in, a_in, a_in, attn_mask=mask, need_weights=False, is_causal=False)
        fused = fused + a_out
        f_in = rn(fused, self.norm_ffn.weight, self.norm_ffn.eps)
        return fused + self.w2(F.silu(self.w1(f_in)) * self.w3(f_in))


class MTPModule(nn.Module):
    """One MTP depth: block, final norm and the shared vocabulary head."""

    def __init__(self, config: dict, depth: int = 1):
        super().__init__()
        self.depth = depth
        self.dim = config["dim"]
        self.vocab_size = config["vocab_size"]
        self.block = MTPBlock(config)
        self.norm = nn.RMSNorm(self.dim, eps=1e-6)
        self.output_head: Optional[nn.Linear] = None

    def set_output_head(self, head: nn.Linear) -> None:
        """Share the main model's vocabulary projection.

        The head is registered as a child module (as in the reference); its
        weight is the main model's, so checkpoint writers drop the duplicate
        key by storage identity.
        """
        self.output_head = head

    def hidden(self, prev_hidden: torch.Tensor, target_emb: torch.Tensor) -> torch.Tensor:
        """Normalised MTP hidden state (input of the shared head)."""
        if prev_hidden.shape != target_emb.shape:
            raise ValueError(f"Shape mismatch: {tuple(prev_hidden.shape)} vs {tuple(target_emb.shape)}")
        h = self.block(prev_hidden, target_emb)
        return norm_ops.rms_norm(h, self.norm.weight, self.norm.eps)

    def forward(self, prev_hidden: torch.Tensor, target_emb: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Return ``(draft logits, normalised hidden)``."""
        if self.output_head is None:
            raise RuntimeError(f"MTPModule(depth={self.depth}): output_head not set.")
        h_norm = self.hidden(prev_hidden, target_emb)
        return self.output_head(h_norm), h_norm


def _mtp_settings(config: dict) -> Tuple[int, float]:
    if "mtp_depth" in config:
        return config["mtp_depth"], config.get("mtp_loss_weight", 0.3)
    sub = config.get("mtp", {})
    return sub.get("depth", 1), sub.get("weight", 0.3)


class MultiTokenPrediction(nn.Module):
    """Main model plus ``depth`` chained MTP predictors sharing embed and head."""

    def __init__(self, config: dict, main_model: nn.Module):
        super().__init__()
        self.main_model = main_model
        self.depth, self.mtp_weight = _mtp_settings(config)
        model_cfg = config.get("model", config)
        self.mtp_modules = nn.ModuleList(MTPModule(model_cfg, d + 1) for d in range(self.depth))
        self.add_module("embed", main_model.embed)
        for m in self.mtp_modules:
            m.set_output_head(main_model.head)

    def mtp_inputs(self, tokens: torch.Tensor, d: int):
        """``(usable, embedding input ids, target ids)`` for MTP depth ``d``."""
        usable = tokens.size(1) - d - 2
        return usable, tokens[:, d + 1:d + 1 + usable], tokens[:, d + 2:d + 2 + usable]

    def forward(self, tokens: torch.Tensor) -> Tuple[torch.Tensor, List[Tuple[torch.Tensor, torch.Tensor]]]:
        """Return main logits and per-depth ``(logits, targets)`` pairs."""
        if tokens.dim() < 2:
            raise ValueError(f"Expected (bsz, seq) tokens, got {tuple(tokens.shape)}")
        main_logits, prev = self.main_model.forward_with_hidden(tokens)
        pairs: List[Tuple[torch.Tensor, torch.Tensor]] = []
        for d, mod in enumerate(self.mtp_modules):
            usable, emb_ids, tgt = self.mtp_inputs(tokens, d)
            if usable <= 0:
                break
            logits, prev = mod(prev[:, :usable], self.embed(emb_ids))
            pairs.append((logits, tgt))
        return main_logits, pairs

    def compute_loss(self, main_logits: torch.Tensor, targets: torch.Tensor,
                     mtp_pairs: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None):
        """Return ``(total, main, mean-MTP)`` losses."""
        main = F.cross_entropy(main_logits.reshape(-1, main_logits.size(-1)), targets.reshape(-1), ignore_index=-100)
        per_depth = [
            F.cross_entropy(lg.reshape(-1, lg.size(-1)), tg.reshape(-1), ignore_index=-100)
            for lg, tg in (mtp_pairs or []) if tg.numel() > 0
        ]
        if not per_depth:
            return main, main, main.new_zeros(())
        mtp = torch.stack(per_depth).mean()
        return main + self.mtp_weight * mtp, main, mtp
