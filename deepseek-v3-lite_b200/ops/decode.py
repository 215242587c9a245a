"""Single-token decode with a per-row cache position.

``Transformer.forward`` decodes every row of a batch at the same position
(reference semantics).  Speculative decoding and continuous batching need
each row at its own position, so this module runs one decode step where row
``b`` is at position ``pos[b]``: its latent is written to cache slot
``pos[b]`` and it attends over ``[0, pos[b]]`` in the absorbed (latent-space)
formulation.  On CUDA the attention is the split-K latent decode kernel
(``csrc/attention.cu``); on CPU it is the masked math below.
"""
from __future__ import annotations

import torch

from . import norm as norm_ops


def _row_rope(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Rotate ``x [B, 1, H, d]`` with per-row complex ``freqs [B, d/2]``."""
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    return torch.view_as_real(xc * freqs.view(x.shape[0], 1, 1, -1)).flatten(-2).to(x.dtype)


def latent_decode_attention(q_lat: torch.Tensor, q_pe: torch.Tensor, kv_cache: torch.Tensor,
                            pe_cache: torch.Tensor, lengths: torch.Tensor, scale: float) -> torch.Tensor:
    """Absorbed decode attention.

    ``q_lat [B, H, R]`` (queries already multiplied by ``W_k``), ``q_pe [B, H, dr]``,
    caches ``[B, S, R]`` / ``[B, S, dr]``, ``lengths [B]`` = number of valid
    cache rows per batch row.  Returns the latent-space output ``[B, H, R]``.
    """
    if q_lat.is_cuda:
        from . import fused
        return fused.latent_decode(q_lat, q_pe, kv_cache, pe_cache, lengths, scale)
    s = kv_cache.shape[1]
    scores = torch.einsum("bhr,bsr->bhs", q_lat.float(), kv_cache.float())
    scores = scores + torch.einsum("bhd,bsd->bhs", q_pe.float(), pe_cache.float())
    valid = torch.arange(s, device=q_lat.device)[None, :] < lengths[:, None]
    scores = (scores * scale).masked_fill(~valid[:, None, :], float("-inf"))
    p = scores.softmax(dim=-1)
    return torch.einsum("bhs,bsr->bhr", p, kv_cache.float()).to(q_lat.dtype)


def mla_decode_rows(attn, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """One MLA decode step for ``x [B, 1, dim]`` with row positions ``pos [B]``."""
    bsz = x.shape[0]
    attn._extend_rope(attn.max_seq_len, x.device)
    attn._ensure_cache(bsz, x.device, x.dtype)
    freqs = attn.freqs_cis[pos]
    q_nope, q_pe = attn._queries(x)
    q_pe = _row_rope(q_pe, freqs)
    latent, k_pe = attn._latents(x)
    k_pe = _row_rope(k_pe.unsqueeze(2), freqs).squeeze(2)
    rows = torch.arange(bsz, device=x.device)
    attn.kv_cache[rows, pos] = latent[:, 0].detach().to(attn.kv_cache.dtype)
    attn.pe_cache[rows, pos] = k_pe[:, 0].detach().to(attn.pe_cache.dtype)
    w_k, w_v = attn._wkv_b_split()
    q_lat = torch.einsum("bhd,hdr->bhr", q_nope[:, 0], w_k.to(q_nope.dtype))
    o_lat = latent_decode_attention(q_lat, q_pe[:, 0], attn.kv_cache[:bsz], attn.pe_cache[:bsz], pos + 1,
                                    attn.softmax_scale)
    o = torch.einsum("bhr,hdr->bhd", o_lat, w_v.to(o_lat.dtype))
    return attn.wo(o.reshape(bsz, 1, -1))


@torch.inference_mode()
def batched_decode_step(model, tokens: torch.Tensor, pos: torch.Tensor):
    """Decode ``tokens [B]`` at positions ``pos [B]``; returns ``(logits [B, V], hidden [B, D])``.

    ``hidden`` is the pre-final-norm state (the MTP input).
    """
    if tokens.is_cuda:
        logits, hid = model.native_inference().decode(tokens.reshape(-1), pos)
        return logits.float(), hid.clone()   # graph outputs are overwritten by the next replay
    h = model.embed(tokens.long()).unsqueeze(1)
    for layer in model.layers:
        x = norm_ops.rms_norm(h, layer.attn_norm.weight, layer.attn_norm.eps)
        h = h + mla_decode_rows(layer.attn, x, pos)
        h = h + layer.ffn(norm_ops.rms_norm(h, layer.ffn_norm.weight, layer.ffn_norm.eps))
    logits = model.head(model.final_hidden(h))[:, 0]
    return logits, h[:, 0]
