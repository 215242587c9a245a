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

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ._native_dispatch import normalize_backend_keys
from .mla import MultiHeadLatentAttention
from .moe import DeepSeekMoE
from ops import norm as norm_ops


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
        for layer in self.layers:
            if self.use_checkpoint and self.training:
                h = torch.utils.checkpoint.checkpoint(layer, h, start_pos, mask, use_cache, use_reentrant=False)
            else:
                h = layer(h, start_pos, mask, use_cache)
        return h

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
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 512, temperature: float = 1.0,
                 top_p: float = 0.9, top_k: int = 0, eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Prefill ``input_ids`` into the latent cache, then decode token by token.

        Stops after ``max_new_tokens``, when every row has produced
        ``eos_token_id``, or when the sequence reaches ``max_seq_len``.
        Training mode is restored afterwards.
        """
        if temperature < 0.0:
            raise ValueError(f"temperature must be >= 0, got {temperature}")
        was_training = self.training
        self.reset_cache()
        self.eval()
        bsz, prompt_len = input_ids.shape
        out = input_ids.clone()
        logits = self.forward(out, start_pos=0, use_cache=True)[:, -1, :]
        done = torch.zeros(bsz, dtype=torch.bool, device=input_ids.device)
        for step in range(max_new_tokens):
            nxt = self._sample(logits, temperature, top_p, top_k)
            out = torch.cat([out, nxt], dim=1)
            if eos_token_id is not None:
                done |= nxt.squeeze(-1) == eos_token_id
                if bool(done.all()):
                    break
            if out.size(1) >= self.max_seq_len:
                break
            logits = self.forward(nxt, start_pos=prompt_len + step, use_cache=True)[:, -1, :]
        if was_training:
            self.train()
        return out

    @staticmethod
    def _sample(logits: torch.Tensor, temperature: float, top_p: float, top_k: int) -> torch.Tensor:
        """Sample one token per row; ``temperature == 0`` is greedy."""
        if temperature == 0.0:
            return logits.argmax(dim=-1, keepdim=True)
        logits = logits / temperature
        if top_k > 0:
            kth = logits.topk(min(top_k, logits.size(-1)), dim=-1).values[:, -1:]
            logits = logits.masked_fill(logits < kth, float("-inf"))
        probs = logits.softmax(dim=-1)
        if top_p >= 1.0:
            return torch.multinomial(probs, 1)
        sp, si = probs.sort(dim=-1, descending=True)
        # Keep every token whose *exclusive* cumulative mass is within top_p.
        sp = sp.masked_fill(sp.cumsum(dim=-1) - sp > top_p, 0.0)
        sp = sp / sp.sum(dim=-1, keepdim=True).clamp(min=1e-10)
        return si.gather(-1, torch.multinomial(sp, 1))


def count_parameters(model: nn.Module) -> Tuple[int, int]:
    """``(total, trainable)`` parameter counts, each tensor counted once."""
    seen, total, trainable = set(), 0, 0
    for p in model.parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        total += p.numel()
        trainable += p.numel() if p.requires_grad else 0
    return total, trainable
