"""MTP-drafted speculative decoding.

``SpeculativeDecoder`` keeps the reference's batch-1 API and acceptance rule
(reference ``inference/speculative.py:12-61``): per step the main model decodes
the last token and samples ``t_main``; a second main pass over ``t_main`` gives
the hidden state the MTP head needs; the MTP head proposes a greedy draft
``t_draft``; the draft is kept iff ``p_main(t_draft) >= tau * p_draft(t_draft)``
(both are softmax probabilities; ``p_main`` is the distribution that produced
``t_main``).  Each step appends one or two tokens.

``BatchedSpeculativeDecoder`` is an extension the reference lacks: the same
rule for a batch of sequences with per-row acceptance and per-row cache
positions, with no host synchronisation inside a step.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from models.mtp import MTPModule
from models.transformer import Transformer


class SpeculativeDecoder:
    """Main-model token plus an MTP draft token, accepted by a probability ratio."""

    def __init__(self, main_model: nn.Module, mtp_module: MTPModule, acceptance_threshold: float = 0.8):
        self.main_model = main_model
        self.mtp = mtp_module
        self.threshold = acceptance_threshold

    @torch.inference_mode()
    def generate_step(self, last_token: torch.Tensor, start_pos: int,
                      temperature: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor, bool]:
        """Decode ``last_token`` at ``start_pos``; return ``(t_main, t_draft, accepted)``."""
        logits = self.main_model(last_token, start_pos=start_pos, use_cache=True)[:, -1, :]
        p_main = torch.softmax(logits.float(), dim=-1)
        t_main = Transformer._sample(logits, temperature, top_p=1.0, top_k=0).squeeze(0)
        _, hidden = self.main_model.forward_with_hidden(t_main.unsqueeze(0), start_pos=start_pos + 1, use_cache=True)
        draft_logits, _ = self.mtp(hidden[:, -1:, :], self.main_model.embed(t_main.unsqueeze(-1)))
        p_draft = torch.softmax(draft_logits[:, -1, :].float(), dim=-1)
        t_draft = p_draft.argmax(dim=-1)
        pm = p_main[0, t_draft[0]].item()
        pd = p_draft[0, t_draft[0]].item()
        return t_main, t_draft, pm >= self.threshold * max(pd, 1e-12)

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 512, temperature: float = 1.0,
                 eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Batch-1 generation; stops at ``max_new_tokens`` new tokens or EOS."""
        out = input_ids.clone()
        if hasattr(self.main_model, "reset_cache"):
            self.main_model.reset_cache()
        self.main_model(out, start_pos=0, use_cache=True)
        produced = 0
        while produced < max_new_tokens:
            t_main, t_draft, ok = self.generate_step(out[:, -1:], start_pos=out.size(1) - 1, temperature=temperature)
            out = torch.cat([out, t_main.unsqueeze(0)], dim=1)
            produced += 1
            if eos_token_id is not None and t_main.item() == eos_token_id:
                break
            if ok and produced < max_new_tokens:
                out = torch.cat([out, t_draft.unsqueeze(0)], dim=1)
                produced += 1
                if eos_token_id is not None and t_draft.item() == eos_token_id:
                    break
        return out


class BatchedSpeculativeDecoder:
    """Speculative decoding for ``B`` sequences at once (greedy main model).

    Rows advance independently: a row whose draft is accepted moves two
    positions, others one.  Sequences are kept in a right-padded buffer with a
    per-row length; the latent cache is indexed by each row's own position.
    The main model is run on all rows at every step (rows that finished keep
    decoding a pad token whose output is discarded), so a step has a fixed
    shape and no host synchronisation.
    """

    def __init__(self, main_model: Transformer, mtp_module: MTPModule, acceptance_threshold: float = 0.8):
        self.main_model = main_model
        self.mtp = mtp_module
        self.threshold = acceptance_threshold

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 64) -> Tuple[torch.Tensor, torch.Tensor]:
        """Return ``(tokens [B, P + max_new_tokens + 1], lengths [B])`` (greedy)."""
        from ops.decode import batched_decode_step
        m = self.main_model
        bsz, plen = input_ids.shape
        cap = plen + max_new_tokens + 1
        if cap > m.max_seq_len:
            raise ValueError(f"prompt + new tokens ({cap}) exceeds max_seq_len {m.max_seq_len}")
        m.reset_cache()
        buf = torch.zeros(bsz, cap, dtype=torch.long, device=input_ids.device)
        buf[:, :plen] = input_ids
        m(input_ids, start_pos=0, use_cache=True)
        lengths = torch.full((bsz,), plen, dtype=torch.long, device=input_ids.device)
        rows = torch.arange(bsz, device=input_ids.device)
        limit = plen + max_new_tokens
        while True:
            active = lengths < limit
            if not bool(active.any()):
                break
            pos = (lengths - 1).clamp(max=cap - 2)
            last = buf[rows, pos]
            logits, _ = batched_decode_step(m, last, pos)
            p_main = torch.softmax(logits.float(), dim=-1)
            t_main = logits.argmax(dim=-1)
            _, hidden = batched_decode_step(m, t_main, pos + 1)
            draft_logits, _ = self.mtp(hidden.unsqueeze(1), m.embed(t_main).unsqueeze(1))
            p_draft = torch.softmax(draft_logits[:, -1].float(), dim=-1)
            t_draft = p_draft.argmax(dim=-1)
            pm = p_main.gather(1, t_draft[:, None]).squeeze(1)
            pd = p_draft.gather(1, t_draft[:, None]).squeeze(1)
            accept = (pm >= self.threshold * pd.clamp(min=1e-12)) & (lengths + 1 < limit) & active
            write1 = torch.where(active, lengths, torch.full_like(lengths, cap - 1))
            buf[rows, write1] = torch.where(active, t_main, buf[rows, write1])
            write2 = torch.where(accept, lengths + 1, torch.full_like(lengths, cap - 1))
            buf[rows, write2] = torch.where(accept, t_draft, buf[rows, write2])
            lengths = lengths + active.long() + accept.long()
        return buf, lengths
