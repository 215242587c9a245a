"""Closed-form memory estimates (no tensors are allocated).

Formulas follow the reference (``utils/memory.py:12-119``): bf16 parameters
(2 B each, tied tensors counted once), fp32 AdamW state (12 B each: master +
two moments), latent KV cache ``B * S * (kv_lora_rank + rope_dim) * 2 B`` per
layer, activations ``24`` (with activation checkpointing) or ``36`` times
``B * S * D * L * 2 B`` (PaLM appendix A), plus a framework overhead of
``min(13.7 GB, max(2 GB, 17% of device memory))`` on CUDA and 2 GB on CPU.

``estimate_sharded_training_gb`` adds what the reference lacks: the per-rank
figure when routed experts are sharded over an expert-parallel group and the
optimizer state over the data-parallel group.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

STATIC_PYTORCH_OVERHEAD_GB = 13.7


def _deduped_numel(model: nn.Module) -> int:
    seen, n = set(), 0
    for p in model.parameters():
        if id(p) not in seen:
            seen.add(id(p))
            n += p.numel()
    return n


def _parameter_bytes(model: nn.Module) -> int:
    return 2 * _deduped_numel(model)


def _optimiser_bytes(model: nn.Module) -> int:
    return 12 * _deduped_numel(model)


def _kv_cache_bytes(model: nn.Module, seq_len: int, batch_size: int, dtype_bytes: int = 2) -> int:
    total = 0
    for layer in getattr(model, "layers", []):
        attn = getattr(layer, "attn", None)
        if attn is None:
            continue
        width = getattr(attn, "kv_lora_rank", 0) + getattr(attn, "qk_rope_head_dim", 0)
        total += batch_size * seq_len * width * dtype_bytes
    return total


def _activation_bytes(seq_len: int, batch_size: int, hidden_dim: int, n_layers: int,
                      grad_checkpoint: bool, dtype_bytes: int = 2) -> int:
    factor = 24 if grad_checkpoint else 36
    return factor * batch_size * seq_len * hidden_dim * n_layers * dtype_bytes


def _infer_dim_n_layers(model: nn.Module):
    embed = getattr(model, "embed", None)
    dim = int(embed.embedding_dim) if embed is not None and hasattr(embed, "embedding_dim") else 0
    layers = getattr(model, "layers", None)
    n = len(layers) if isinstance(layers, nn.ModuleList) else 0
    return dim, n


def _detect_overhead_gb() -> float:
    if not torch.cuda.is_available():
        return 2.0
    total = torch.cuda.get_device_properties(0).total_memory / 1024 ** 3
    return min(STATIC_PYTORCH_OVERHEAD_GB, max(2.0, 0.17 * total))


def estimate_model_memory_gb(model: nn.Module, seq_len: int, batch_size: int, grad_checkpoint: bool = True,
                             overhead_gb=None, dtype_bytes: int = 2, inference: bool = False) -> float:
    """Estimated device memory in GB for training (default) or inference."""
    if overhead_gb is None:
        overhead_gb = _detect_overhead_gb()
    dim, n_layers = _infer_dim_n_layers(model)
    total = _parameter_bytes(model) + _kv_cache_bytes(model, seq_len, batch_size, dtype_bytes)
    if not inference:
        total += _optimiser_bytes(model) + _activation_bytes(seq_len, batch_size, dim, n_layers,
                                                              grad_checkpoint, dtype_bytes)
    return total / 1024 ** 3 + overhead_gb


def assert_fits_in_available_gpu(estimate_gb: float, safety_margin_gb: float = 0.0) -> None:
    """Raise ``RuntimeError`` if ``estimate_gb`` exceeds device 0's memory minus a margin."""
    if not torch.cuda.is_available():
        return
    avail = torch.cuda.get_device_properties(0).total_memory / 1024 ** 3
    if estimate_gb > avail - safety_margin_gb:
        raise RuntimeError(f"estimate {estimate_gb:.2f} GB exceeds available {avail:.2f} GB "
                           f"minus safety margin {safety_margin_gb:.2f} GB")


def estimate_sharded_training_gb(model: nn.Module, seq_len: int, batch_size: int, ep_size: int = 1,
                                 dp_size: int = 1, overhead_gb: float = 2.0, moments_sharded: bool = False) -> float:
    """Per-rank training memory with routed experts (weights, gradients and
    AdamW moments) split over ``ep_size`` ranks, as ``parallel.shard_experts``
    trains.  The moments of the replicated parameters are full-size on every
    rank, as the peer-memory data-parallel step keeps them; with
    ``moments_sharded`` they are counted split over ``dp_size`` ranks instead
    (ZeRO-1 style)."""
    expert_params, dense_params, seen = 0, 0, set()
    for name, p in model.named_parameters():
        if id(p) in seen:
            continue
        seen.add(id(p))
        if ".experts." in name:
            expert_params += p.numel()
        else:
            dense_params += p.numel()
    local = dense_params + expert_params / max(1, ep_size)
    # fp32 master + fp32 grad + bf16 shadow per local parameter; moments sharded.
    param_bytes = local * (4 + 4 + 2)
    dense_moment_share = dense_params / max(1, dp_size) if moments_sharded else dense_params
    moment_bytes = 8 * (dense_moment_share + expert_params / max(1, ep_size))
    dim, n_layers = _infer_dim_n_layers(model)
    act = _activation_bytes(seq_len, batch_size, dim, n_layers, False)
    return (param_bytes + moment_bytes + act) / 1024 ** 3 + overhead_gb


def expert_sharding_hint(model: nn.Module, seq_len: int, batch_size: int, world_size: int, ep_size: int,
                         shard_experts: bool, device_gb: float) -> Optional[str]:
    """A warning when this run's per-rank training state will not fit
    ``device_gb`` but would with routed experts sharded over the ranks (or
    ``None``).  ``ep_size`` 0 means all ranks."""
    ep = world_size if ep_size in (0, world_size) else 1
    shards = ep if (shard_experts and ep > 1) else 1
    need = estimate_sharded_training_gb(model, seq_len, batch_size, ep_size=shards, dp_size=world_size)
    if need <= device_gb:
        return None
    if shards == 1 and world_size > 1:
        with_shards = estimate_sharded_training_gb(model, seq_len, batch_size, ep_size=world_size, dp_size=world_size)
        if with_shards <= device_gb:
            return (f"estimated {need:.0f} GB per rank exceeds the {device_gb:.0f} GB device; with routed experts "
                    f"sharded over the {world_size} ranks it is ~{with_shards:.0f} GB "
                    f"(parallel: {{ep_size: 0, shard_experts: true}})")
    return (f"estimated {need:.0f} GB per rank exceeds the {device_gb:.0f} GB device (more ranks with sharded "
            f"experts, or a smaller micro-batch)")
