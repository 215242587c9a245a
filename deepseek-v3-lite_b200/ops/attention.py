"""MLA attention cores: materialised-K/V and absorbed formulations.

Both take rotated ``q_pe``/``ctx_pe`` and the RMS-normalised latent ``ctx_kv``
and return ``[B, Sq, H, dv]`` before the output projection.  Semantics follow
reference ``models/mla.py:150-180``:

* materialised: ``K_nope = ctx_kv @ W_k^T``, ``V = ctx_kv @ W_v^T`` per head, then
  ``softmax(scale * [q_nope|q_pe] . [K_nope|k_pe]^T + mask) @ V``;
* absorbed: ``scores = (q_nope @ W_k) . ctx_kv^T + q_pe . ctx_pe^T``, softmax in
  fp32, ``(P @ ctx_kv) @ W_v^T``.

The causal rule is by global position: query ``i`` (at ``q_offset + i``) sees
key ``j`` iff ``q_offset + i >= j`` (reference ``models/transformer.py:63-78``).
These functions are the CPU implementations and the numerics oracle for the
CUDA kernels in ``csrc/attention.cu`` (reached through ``ops.fused``).
"""
from __future__ import annotations

from typing import Optional

import torch


def causal_additive_mask(sq: int, sk: int, q_offset: int, device=None) -> torch.Tensor:
    q = torch.arange(sq, device=device)[:, None] + q_offset
    k = torch.arange(sk, device=device)[None, :]
    zero = torch.zeros((), device=device)
    return torch.where(q >= k, zero, torch.full((), float("-inf"), device=device))


def _softmax_weighted(scores: torch.Tensor, scale: float, mask: Optional[torch.Tensor], out_dtype) -> torch.Tensor:
    scores = scores * scale
    if mask is not None:
        scores = scores + mask
    return scores.softmax(dim=-1, dtype=torch.float32).to(out_dtype)


def mla_materialized(q_nope, q_pe, ctx_kv, ctx_pe, w_k, w_v, scale: float, causal: bool = True,
                     q_offset: int = 0, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention over K/V materialised from the latent; returns ``[B, Sq, H, dv]``."""
    sq, sk = q_nope.shape[1], ctx_kv.shape[1]
    if mask is None and causal and sq > 1:
        mask = causal_additive_mask(sq, sk, q_offset, q_nope.device)
    k_nope = torch.einsum("bsr,hdr->bhsd", ctx_kv, w_k.to(ctx_kv.dtype))
    v = torch.einsum("bsr,hdr->bhsd", ctx_kv, w_v.to(ctx_kv.dtype))
    h = q_nope.shape[2]
    q = torch.cat([q_nope, q_pe], dim=-1).transpose(1, 2)                       # [B,H,Sq,dqk]
    k = torch.cat([k_nope, ctx_pe.unsqueeze(1).expand(-1, h, -1, -1).to(k_nope.dtype)], dim=-1)
    p = _softmax_weighted(q.float() @ k.float().transpose(-1, -2), scale, mask, v.dtype)
    return (p @ v).transpose(1, 2)


def mla_absorbed(q_nope, q_pe, ctx_kv, ctx_pe, w_k, w_v, scale: float, causal: bool = True,
                 q_offset: int = 0, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention in the latent space (weights absorbed); returns ``[B, Sq, H, dv]``."""
    sq, sk = q_nope.shape[1], ctx_kv.shape[1]
    if mask is None and causal and sq > 1:
        mask = causal_additive_mask(sq, sk, q_offset, q_nope.device)
    q_lat = torch.einsum("bshd,hdr->bhsr", q_nope, w_k.to(q_nope.dtype))       # [B,H,Sq,R]
    scores = q_lat.float() @ ctx_kv.float().unsqueeze(1).transpose(-1, -2)
    scores = scores + q_pe.transpose(1, 2).float() @ ctx_pe.float().unsqueeze(1).transpose(-1, -2)
    p = _softmax_weighted(scores, scale, mask, q_nope.dtype)
    out_lat = p @ ctx_kv.unsqueeze(1).to(p.dtype)                               # [B,H,Sq,R]
    out = torch.einsum("bhsr,hdr->bhsd", out_lat, w_v.to(out_lat.dtype))
    return out.transpose(1, 2)


def mla_attention_reference(q_nope, q_pe, ctx_kv, ctx_pe, wkv_b_k, wkv_b_v, softmax_scale: float,
                            is_causal: bool = True, q_start: int = 0) -> torch.Tensor:
    """Oracle with the reference kernel's argument layout (heads before sequence).

    Mirrors the signature of the reference's CPU oracle
    (``models/mla_triton.py:28-67``): ``q_nope``/``q_pe`` are ``[B, H, Sq, d]``;
    returns ``[B, Sq, H, dv]``.
    """
    return mla_materialized(q_nope.transpose(1, 2), q_pe.transpose(1, 2), ctx_kv, ctx_pe, wkv_b_k, wkv_b_v,
                            softmax_scale, causal=is_causal, q_offset=q_start)
