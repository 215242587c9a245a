"""Multi-head Latent Attention (MLA) with a latent KV cache.

Behaviour follows the reference layer (reference ``models/mla.py:14-218``):

* queries come from ``wq`` or from the LoRA chain ``wq_a -> q_norm -> wq_b``;
* ``wkv_a`` produces the compressed latent (``kv_lora_rank``) plus one shared
  RoPE key of ``qk_rope_head_dim``; the latent is RMS-normalised;
* decoupled RoPE (interleaved pairs, fp32) is applied to ``q_pe`` and ``k_pe``;
* ``wkv_b`` is viewed as ``[H, dn + dv, R]`` with the K rows first;
* the cache stores the *post-norm* latent and the *post-RoPE* ``k_pe``;
* softmax scale ``(dn + dr) ** -0.5``, times ``mscale ** 2`` only when
  ``max_seq_len > 4096``; YaRN changes ``mscale`` only (``rope_factor > 1``).

Two formulations are offered (see ``_native_dispatch``): materialised K/V
(``sdpa``/``native``) and absorbed (``manual``).  On CUDA both run on the
hand-written kernels in ``ops.attention``; on CPU they run as PyTorch math.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ops import attention as attn_ops
from ops import norm as norm_ops
from ops import rope as rope_ops


class MultiHeadLatentAttention(nn.Module):
    """MLA layer with low-rank KV compression, decoupled RoPE and a latent cache."""

    def __init__(self, config: dict, layer_idx: int = 0):
        super().__init__()
        self.layer_idx = layer_idx
        self.attn_impl = config.get("attn_impl", "sdpa")
        if self.attn_impl == "triton":
            self.attn_impl = "native"
        self.dim = config["dim"]
        self.n_heads = config["n_heads"]
        self.n_local_heads = self.n_heads
        self.q_lora_rank = config["q_lora_rank"]
        self.kv_lora_rank = config["kv_lora_rank"]
        self.qk_nope_head_dim = config["qk_nope_head_dim"]
        self.qk_rope_head_dim = config["qk_rope_head_dim"]
        self.v_head_dim = config["v_head_dim"]
        self.qk_head_dim = self.qk_nope_head_dim + self.qk_rope_head_dim
        self.max_seq_len = config["max_seq_len"]
        self.rope_theta = config["rope_theta"]
        self.rope_factor = config.get("rope_factor", 1.0)
        base_mscale = config.get("mscale", 1.0)
        # YaRN only rescales the softmax temperature here; frequencies are untouched.
        self.mscale = (0.1 * base_mscale * math.log(self.rope_factor) + 1.0) if self.rope_factor > 1.0 else base_mscale
        scale = self.qk_head_dim ** -0.5
        self.softmax_scale = scale * self.mscale ** 2 if self.max_seq_len > 4096 else scale

        H = self.n_heads
        if self.q_lora_rank > 0:
            self.wq_a = nn.Linear(self.dim, self.q_lora_rank, bias=False)
            self.q_norm = nn.RMSNorm(self.q_lora_rank, eps=1e-6)
            self.wq_b = nn.Linear(self.q_lora_rank, H * self.qk_head_dim, bias=False)
        else:
            self.wq = nn.Linear(self.dim, H * self.qk_head_dim, bias=False)
        self.wkv_a = nn.Linear(self.dim, self.kv_lora_rank + self.qk_rope_head_dim, bias=False)
        self.kv_norm = nn.RMSNorm(self.kv_lora_rank, eps=1e-6)
        self.wkv_b = nn.Linear(self.kv_lora_rank, H * (self.qk_nope_head_dim + self.v_head_dim), bias=False)
        self.wo = nn.Linear(H * self.v_head_dim, self.dim, bias=False)

        self._cache_batch = 0
        self.kv_cache: Optional[torch.Tensor] = None
        self.pe_cache: Optional[torch.Tensor] = None
        self._rope_seq_len = 0
        self.register_buffer(
            "freqs_cis", torch.empty(0, self.qk_rope_head_dim // 2, dtype=torch.complex64), persistent=False
        )

    # ------------------------------------------------------------------ rope
    def _extend_rope(self, seq_len: int, device: torch.device) -> None:
        """Grow the RoPE table geometrically (x2, at least 64), capped at max_seq_len."""
        if seq_len <= self._rope_seq_len and self.freqs_cis.device == torch.device(device):
            return
        target = min(max(seq_len, self._rope_seq_len * 2, 64), self.max_seq_len)
        self.freqs_cis = rope_ops.rope_table(target, self.qk_rope_head_dim, self.rope_theta, device)
        self._rope_seq_len = target

    def _apply_rope(self, x: torch.Tensor, start_pos: int, seqlen: int) -> torch.Tensor:
        return rope_ops.apply_rope_complex(x, self.freqs_cis[start_pos:start_pos + seqlen])

    # ----------------------------------------------------------------- cache
    def _ensure_cache(self, bsz: int, device: torch.device, dtype: torch.dtype) -> None:
        """Allocate (or grow) the latent cache to ``max(bsz, 2*old, 16)`` rows."""
        fresh = (
            self.kv_cache is None
            or bsz > self._cache_batch
            or self.kv_cache.device != torch.device(device)
            or self.kv_cache.dtype != dtype
        )
        if not fresh:
            return
        rows = max(bsz, self._cache_batch * 2, 16)
        self.kv_cache = torch.zeros(rows, self.max_seq_len, self.kv_lora_rank, device=device, dtype=dtype)
        self.pe_cache = torch.zeros(rows, self.max_seq_len, self.qk_rope_head_dim, device=device, dtype=dtype)
        self._cache_batch = rows

    def reset_cache(self) -> None:
        """Drop the cached latents and RoPE keys."""
        self.kv_cache = None
        self.pe_cache = None
        self._cache_batch = 0

    # ------------------------------------------------------------ projections
    def _wkv_b_split(self):
        w = self.wkv_b.weight.view(self.n_heads, self.qk_nope_head_dim + self.v_head_dim, self.kv_lora_rank)
        return w[:, :self.qk_nope_head_dim], w[:, self.qk_nope_head_dim:]

    def _queries(self, x: torch.Tensor):
        if self.q_lora_rank > 0:
            q = self.wq_b(norm_ops.rms_norm(self.wq_a(x), self.q_norm.weight, self.q_norm.eps))
        else:
            q = self.wq(x)
        bsz, seqlen, _ = x.shape
        q = q.view(bsz, seqlen, self.n_heads, self.qk_head_dim)
        return q.split([self.qk_nope_head_dim, self.qk_rope_head_dim], dim=-1)

    def _latents(self, x: torch.Tensor):
        kv_a = self.wkv_a(x)
        latent, k_pe = kv_a.split([self.kv_lora_rank, self.qk_rope_head_dim], dim=-1)
        return norm_ops.rms_norm(latent, self.kv_norm.weight, self.kv_norm.eps), k_pe

    # ---------------------------------------------------------------- forward
    def forward(self, x: torch.Tensor, start_pos: int = 0, mask: Optional[torch.Tensor] = None,
                use_cache: bool = True) -> torch.Tensor:
        """Attend over ``x`` of shape ``[B, S, dim]``; returns ``[B, S, dim]``.

        ``mask`` is the additive causal mask built by the Transformer (``None``
        for single-token decode).  With ``use_cache`` the latents are written to
        the cache at ``[start_pos, start_pos + S)`` and attention spans the
        whole cached prefix ``[0, start_pos + S)``.
        """
        bsz, seqlen, _ = x.shape
        end_pos = start_pos + seqlen
        if end_pos > self.max_seq_len:
            raise RuntimeError(f"Layer {self.layer_idx}: end_pos {end_pos} exceeds max_seq_len {self.max_seq_len}")
        self._extend_rope(end_pos, x.device)
        if use_cache:
            self._ensure_cache(bsz, x.device, x.dtype)

        q_nope, q_pe = self._queries(x)
        q_pe = self._apply_rope(q_pe, start_pos, seqlen)
        latent, k_pe = self._latents(x)
        k_pe = self._apply_rope(k_pe.unsqueeze(2), start_pos, seqlen).squeeze(2)

        if use_cache:
            self.kv_cache[:bsz, start_pos:end_pos] = latent.detach()
            self.pe_cache[:bsz, start_pos:end_pos] = k_pe.detach()
            ctx_kv = self.kv_cache[:bsz, :end_pos]
            ctx_pe = self.pe_cache[:bsz, :end_pos]
        else:
            ctx_kv, ctx_pe = latent, k_pe

        w_k, w_v = self._wkv_b_split()
        # The causal offset of the queries inside the attended window.
        causal = mask is not None
        q_offset = start_pos if use_cache else 0
        if self.attn_impl == "manual":
            out = attn_ops.mla_absorbed(q_nope, q_pe, ctx_kv, ctx_pe, w_k, w_v, self.softmax_scale,
                                        causal=causal, q_offset=q_offset, mask=mask)
        else:
            out = attn_ops.mla_materialized(q_nope, q_pe, ctx_kv, ctx_pe, w_k, w_v, self.softmax_scale,
                                            causal=causal, q_offset=q_offset, mask=mask)
        return self.wo(out.reshape(bsz, seqlen, self.n_heads * self.v_head_dim))
