"""RMSNorm entry points.

``y = x / sqrt(mean(x^2) + eps) * w`` (reference uses ``nn.RMSNorm`` with
``eps=1e-6`` everywhere: ``models/transformer.py:29-31``, ``models/mla.py:45``).
CPU tensors use ``torch.nn.functional.rms_norm``; the CUDA kernels live in
``csrc/norm_rope.cu`` and are reached through ``ops.fused``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMS-normalise the last dimension of ``x`` and scale by ``weight``."""
    if eps is None:
        eps = 1e-6
    return F.rms_norm(x, (x.shape[-1],), weight, eps)
