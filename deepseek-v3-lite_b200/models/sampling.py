"""Batched token sampling without host synchronisation.

Rule (the reference's ``Transformer._sample``, ``models/transformer.py:165-184``):

* ``temperature == 0`` picks the arg-max;
* otherwise the logits are divided by ``temperature``; ``top_k > 0`` keeps the
  logits at or above the k-th largest; ``top_p < 1`` keeps, in descending
  probability order, every token whose *exclusive* cumulative probability is
  at most ``top_p`` (so the most likely token always survives); one token is
  drawn from the renormalised survivors.

The draw is an exponential race: with independent ``E_i ~ Exp(1)``,
``argmax_i p_i / E_i`` is distributed as ``Categorical(p / sum(p))``.  It
needs neither renormalisation nor ``torch.multinomial`` (which checks its
input on the host), filtered tokens (``p_i = 0``) can never win, and every
row of a batch is drawn by the same few kernels.  Both the eager
``Transformer.generate`` and the native decode loops use this function.
"""
from __future__ import annotations

from typing import Optional

import torch


def filtered_probs(logits: torch.Tensor, temperature: float, top_p: float = 1.0, top_k: int = 0) -> torch.Tensor:
    """Probabilities after temperature, top-k and top-p filtering (not renormalised), fp32 ``[B, V]``."""
    z = logits.float() / temperature
    if top_k > 0:
        k = min(int(top_k), z.size(-1))
        floor = torch.topk(z, k, dim=-1).values[..., -1:]
        z = torch.where(z >= floor, z, torch.full_like(z, float("-inf")))
    p = torch.softmax(z, dim=-1)
    if top_p < 1.0:
        desc, order = torch.sort(p, dim=-1, descending=True)
        before = torch.cumsum(desc, dim=-1) - desc              # mass strictly ahead of each token
        keep_sorted = before <= top_p
        keep = torch.zeros_like(keep_sorted).scatter_(-1, order, keep_sorted)
        p = p * keep
    return p


def sample_tokens(logits: torch.Tensor, temperature: float, top_p: float = 1.0, top_k: int = 0,
                  generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """One token id per row of ``logits [B, V]`` as ``[B, 1]`` int64."""
    if temperature == 0.0:
        return torch.argmax(logits, dim=-1, keepdim=True)
    p = filtered_probs(logits, temperature, top_p, top_k)
    race = torch.empty_like(p).exponential_(1.0, generator=generator)
    race.clamp_(min=torch.finfo(race.dtype).tiny)               # a zero draw would turn p = 0 into NaN
    return torch.argmax(p / race, dim=-1, keepdim=True)
