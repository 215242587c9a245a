"""Decoupled rotary position embedding (RoPE) for MLA.

Semantics (reference ``models/mla.py:59-75``): the rotary dimension is split
into interleaved pairs ``(x[2i], x[2i+1])`` treated as one complex number and
multiplied by ``exp(1j * t * theta ** (-2i / d))`` in fp32; the result is cast
back to the input dtype.  The table covers positions ``[0, n)``.

CUDA tensors go through the fused kernel in ``csrc/norm_rope.cu`` (the rotation
is fused into the QKV split that feeds attention); CPU tensors use the complex
multiply below.
"""
from __future__ import annotations

import torch


def inv_frequencies(dim: int, theta: float, device=None) -> torch.Tensor:
    """``theta ** (-2i/dim)`` for ``i < dim/2`` in fp32."""
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32, device=device) / dim))


def rope_table(n: int, dim: int, theta: float, device=None) -> torch.Tensor:
    """Complex64 table ``[n, dim/2]`` of unit rotations for positions ``0..n-1``."""
    angles = torch.outer(torch.arange(n, dtype=torch.float32, device=device), inv_frequencies(dim, theta, device))
    return torch.polar(torch.ones_like(angles), angles)


def apply_rope_complex(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Rotate ``x`` of shape ``[B, S, H, d]`` by ``freqs`` ``[S, d/2]`` (complex)."""
    b, s = x.shape[0], x.shape[1]
    xc = torch.view_as_complex(x.float().reshape(*x.shape[:-1], -1, 2))
    out = torch.view_as_real(xc * freqs.view(1, s, 1, -1)).flatten(-2)
    return out.to(x.dtype)


def rope_cos_sin(n: int, dim: int, theta: float, device=None):
    """fp32 ``cos`` and ``sin`` tables ``[n, dim/2]`` used by the CUDA kernels."""
    angles = torch.outer(torch.arange(n, dtype=torch.float32, device=device), inv_frequencies(dim, theta, device))
    return torch.cos(angles).contiguous(), torch.sin(angles).contiguous()
