"""DeepSeek-V3-Lite decoder: embedding -> N x (MLA + dense/MoE FFN) -> norm -> head.

Public surface and semantics match the reference (``models/transformer.py``):
``Transformer(config, use_checkpoint)`` accepts a flat model dict or one with a
``model`` section; ``forward`` returns ``[B, S, vocab]`` logits,
``forward_with_hidden`` also returns the pre-final-norm hidden state used by
MTP, ``generate`` samples autoregressively over the latent cache, and
``_sample`` implements temperature / top-k / top-p (exclusive cumulative mass)
sampling.  Layers ``< n_dense_layers`` use a dense SwiGLU FFN, the rest MoE.

This module is the eager, module-by-module path (CPU oracle and inference).
The B200 training step runs the same parameters through the fused CUDA
engine in ``ops.engine``.
"""
from __future__ import annotations

import functools
from typing import Optional, Tuple

import torch
import torch.utils.checkpoint
import torch.nn as nn
import torch.nn.functional as F

from ._native_dispatch import normalize_backend_keys
from .mla import MultiHeadLatentAttention
from .moe import DeepSeekMoE
from .sampling import sample_tokens
from ops import norm as norm_ops


def _direct(block: nn.Module, *args):
    return block(*args)


def _recomputed(block: nn.Module, *args):
    return torch.utils.checkpoint.checkpoint(block, *args, use_reentrant=False)


class SwiGLUFFN(nn.Module):
    """Dense gated FFN ``w2(silu(w1 x) * w3 x)``."""

    def __init__(self, dim: int, inter_dim: int):
        super().__init__()
        self.w1 = nn.Linear(dim, inter_dim, bias=False)
        self.w2 = nn.Linear(inter_dim, dim, bias=False)
        self.w3 = nn.Linear(dim, inter_dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class TransformerBlock(nn.Module):
    """Pre-norm residual block: MLA, then a dense or MoE FFN."""

    def __init__(self, layer_id: int, config: dict):
        super().__init__()
        self.layer_id = layer_id
        self.dim = config["dim"]
        self.n_dense_layers = config["n_dense_layers"]
        self.attn_norm = nn.RMSNorm(self.dim, eps=1e-6)
        self.attn = MultiHeadLatentAttention(config, layer_id)
        self.ffn_norm = nn.RMSNorm(self.dim, eps=1e-6)
        self.ffn = SwiGLUFFN(self.dim, config["inter_dim"]) if layer_id < self.n_dense_layers else DeepSeekMoE(config)

    def forward(self, x: torch.Tensor, start_pos: int = 0, mask: Optional[torch.Tensor] = None,
                use_cache: bool = True) -> torch.Tensor:
        rn = norm_ops.rms_norm
        x = x + self.attn(rn(x, self.attn_norm.weight, self.attn_norm.eps), start_pos, mask, use_cache)
        return x + self.ffn(rn(x, self.ffn_norm.weight, self.ffn_norm.eps))


class Transformer(nn.Module):
    """DeepSeek-V3-style decoder with MLA attention and DeepSeekMoE FFNs."""

    def __init__(self, config: dict, use_checkpoint: bool = False):
        super().__init__()
        cfg = config.get("model", config)
        normalize_backend_keys(cfg)
        self.config = cfg
        self.use_checkpoint = use_checkpoint
        self.max_seq_len = cfg["max_seq_len"]
        self.embed = nn.Embedding(cfg["vocab_size"], cfg["dim"])
        nn.init.normal_(self.embed.weight, std=0.006)
        self.layers = nn.ModuleList(TransformerBlock(i, cfg) for i in range(cfg["n_layers"]))
        self.norm = nn.RMSNorm(cfg["dim"], eps=1e-6)
        self.weight_tying = cfg.get("weight_tying", False)
        self.head = nn.Linear(cfg["dim"], cfg["vocab_size"], bias=False)
        if self.weight_tying:
            self.head.weight = self.embed.weight
        self._mask_cache: Optional[torch.Tensor] = None
        self._mask_key = None

    # ----------------------------------------------------------------- masks
    def _build_causal_mask(self, seqlen: int, kv_len: int, start_pos: int, device) -> torch.Tensor:
        """Additive ``[1, 1, S, kv_len]`` mask, causal by global position (cached)."""
        key = (seqlen, kv_len, start_pos, torch.device(device))
        if self._mask_cache is None or self._mask_key != key:
            q = torch.arange(seqlen, device=device).unsqueeze(1) + start_pos
            k = torch.arange(kv_len, device=device).unsqueeze(0)
            m = torch.zeros(seqlen, kv_len, device=device).masked_fill(q < k, float("-inf"))
            self._mask_cache = m.view(1, 1, seqlen, kv_len)
            self._mask_key = key
        return self._mask_cache

    def _run_layers(self, h: torch.Tensor, start_pos: int, mask: Optional[torch.Tensor], use_cache: bool) -> torch.Tensor:
        """Apply the blocks in order; with activation checkpointing on (training only) each block is recomputed in backward."""
        call = _recomputed if (self.use_checkpoint and self.training) else _direct
        return functools.reduce(lambda x, block: call(block, x, start_pos, mask, use_cache), self.layers, h)

    def reset_cache(self) -> None:
        """Clear the latent caches of every layer."""
        for layer in self.layers:
            layer.attn.reset_cache()

    def moe_layers(self):
        """Iterate over the MoE FFNs (for bias updates and diagnostics)."""
        for layer in self.layers:
            if isinstance(layer.ffn, DeepSeekMoE):
                yield layer.ffn

    def _trunk(self, tokens: torch.Tensor, start_pos: int, use_cache: bool) -> torch.Tensor:
        if tokens.dtype != torch.long:
            tokens = tokens.long()
        seqlen = tokens.size(1)
        h = self.embed(tokens)
        mask = None
        if seqlen > 1:
            kv_len = start_pos + seqlen if use_cache else seqlen
            mask = self._build_causal_mask(seqlen, kv_len, start_pos if use_cache else 0, tokens.device)
        return self._run_layers(h, start_pos, mask, use_cache)

    def final_hidden(self, h: torch.Tensor) -> torch.Tensor:
        """Final RMSNorm applied to a trunk hidden state."""
        return norm_ops.rms_norm(h, self.norm.weight, self.norm.eps)

    def native_inference(self):
        """The sm_100a inference engine bound to this model (created on first use).

        Cached, gradient-free calls on CUDA tensors with ``use_cache=True`` run
        on it (prefill + latent-cache decode); training and CPU calls use the
        module path below.
        """
        dev = self.embed.weight.device
        eng = self.__dict__.get("_infer_engine")
        if eng is None or eng.device != dev:
            from ops.infer import InferenceEngine
            eng = InferenceEngine(self)
            self.__dict__["_infer_engine"] = eng
        return eng

    def _use_native(self, tokens: torch.Tensor, use_cache: bool) -> bool:
        return tokens.is_cuda and use_cache and not torch.is_grad_enabled()

    def forward(self, tokens: torch.Tensor, start_pos: int = 0, use_cache: bool = True) -> torch.Tensor:
        """Logits ``[B, S, vocab]``; ``start_pos`` is the cache offset of ``tokens``."""
        if self._use_native(tokens, use_cache):
            eng = self.native_inference()
            if tokens.shape[1] == 1:   # decode step: CUDA-graph replay
                pos = torch.full((tokens.shape[0],), start_pos, dtype=torch.int32, device=tokens.device)
                return eng.decode(tokens[:, 0], pos)[0].float().unsqueeze(1)
            return eng.forward(tokens, start_pos=start_pos)[0].float()
        return self.head(self.final_hidden(self._trunk(tokens, start_pos, use_cache)))

    def forward_with_hidden(self, tokens: torch.Tensor, start_pos: int = 0,
                            use_cache: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
        """``(logits, pre-final-norm hidden)``; the hidden feeds MTP."""
        if self._use_native(tokens, use_cache):
            eng = self.native_inference()
            if tokens.shape[1] == 1:
                pos = torch.full((tokens.shape[0],), start_pos, dtype=torch.int32, device=tokens.device)
                logits, h = eng.decode(tokens[:, 0], pos)
                return logits.float().unsqueeze(1), h.unsqueeze(1)
            logits, h = eng.forward(tokens, start_pos=start_pos, want_hidden=True)
            return logits.float(), h
        h = self._trunk(tokens, start_pos, use_cache)
        return self.head(self.final_hidden(h)), h

    # ------------------------------------------------------------- generation
    @torch.inference_mode()
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 512, temperature: float = 1.0,
                 top_p: float = 0.9, top_k: int = 0, eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Prefill ``input_ids`` into the latent cache, then decode one token per step.

        Stops after ``max_new_tokens``, once every row has produced
        ``eos_token_id``, or when the sequence reaches ``max_seq_len`` (at
        least one token is always produced).  The caches are reset first and
        the training mode is restored afterwards.  Tokens are written into one
        preallocated ``[B, prompt + budget]`` buffer; the only per-step host
        read is the end-of-sequence test when ``eos_token_id`` is given.
        """
        if temperature < 0.0:
            raise ValueError(f"temperature must be >= 0, got {temperature}")
        bsz, prompt_len = input_ids.shape
        budget = min(max_new_tokens, max(1, self.max_seq_len - prompt_len)) if max_new_tokens > 0 else 0
        out = torch.empty(bsz, prompt_len + budget, dtype=input_ids.dtype, device=input_ids.device)
        out[:, :prompt_len] = input_ids
        restore = self.training
        self.reset_cache()
        self.eval()
        try:
            written = self._decode_into(out, prompt_len, budget, temperature, top_p, top_k, eos_token_id)
        finally:
            self.train(restore)
        return out[:, :prompt_len + written].clone()

    def _decode_into(self, out: torch.Tensor, prompt_len: int, budget: int, temperature: float, top_p: float,
                     top_k: int, eos_token_id: Optional[int]) -> int:
        """Fill ``out[:, prompt_len:prompt_len + budget]``; returns how many columns were written."""
        if budget == 0:
            return 0
        alive = None if eos_token_id is None else torch.ones(out.size(0), dtype=torch.bool, device=out.device)
        logits = self.forward(out[:, :prompt_len], start_pos=0, use_cache=True)[:, -1]
        for i in range(budget):
            tok = self._sample(logits, temperature, top_p, top_k)
            out[:, prompt_len + i] = tok[:, 0]
            if alive is not None:
                alive &= tok[:, 0] != eos_token_id
                if not bool(alive.any()):
                    return i + 1
            if i + 1 < budget:
                logits = self.forward(tok, start_pos=prompt_len + i, use_cache=True)[:, -1]
        return budget

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float, top_k: int) -> torch.Tensor:
        """One token per row (``[B, 1]``); ``temperature == 0`` is greedy (``models/sampling.py``)."""
        return sample_tokens(logits, temperature, top_p, top_k)


def count_parameters(model: nn.Module) -> Tuple[int, int]:
    """``(total, trainable)`` element counts; a tied tensor counts once.

    ``nn.Module.parameters()`` already yields a shared ``Parameter`` (the tied
    embedding / head) a single time, which is the deduplication the
    reference applies by tensor identity.
    """
    params = list(model.parameters())
    return sum(p.numel() for p in params), sum(p.numel() for p in params if p.requires_grad)
