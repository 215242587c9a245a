"""Import surface of the reference's ``models/moe_triton.py`` for code written
against it: ``HAS_TRITON``, ``grouped_moe_pytorch`` and
``triton_grouped_moe_dispatch`` (reference ``models/moe_triton.py:28-52``,
``:504``).

This build has no Triton kernels.  Routed experts run on its grouped tcgen05
GEMMs whenever the model trains or decodes on CUDA, whatever ``moe_dispatch``
says, so ``HAS_TRITON`` is always False and ``triton_grouped_moe_dispatch``
raises ``ImportError``.  ``grouped_moe_pytorch`` is a plain PyTorch oracle of
a grouped SwiGLU expert layer.
"""
import torch
import torch.nn.functional as F

HAS_TRITON = False

__all__ = ["HAS_TRITON", "grouped_moe_pytorch", "triton_grouped_moe_dispatch"]


def grouped_moe_pytorch(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor,
                        offsets: torch.Tensor, gate_weights: torch.Tensor) -> torch.Tensor:
    """Rows ``offsets[e]:offsets[e+1]`` of ``x`` ``[T, D]`` (sorted by expert)
    go through expert ``e``: ``w2[e] (silu(w1[e] x) * w3[e] x)``, scaled by
    their ``gate_weights``; ``w1``, ``w3`` ``[E, I, D]``, ``w2`` ``[E, D, I]``.
    Returns ``[T, D]`` in ``x``'s dtype (rows outside every range are zero)."""
    y = torch.zeros_like(x)
    bounds = offsets.tolist()
    for e in range(w1.shape[0]):
        lo, hi = int(bounds[e]), int(bounds[e + 1])
        if hi <= lo:
            continue
        rows = x[lo:hi]
        h = F.silu(rows @ w1[e].t()) * (rows @ w3[e].t())
        y[lo:hi] = (h @ w2[e].t()) * gate_weights[lo:hi].unsqueeze(-1).to(x.dtype)
    return y


def triton_grouped_moe_dispatch(*args, **kwargs):
    raise ImportError("triton kernels are not part of this build: routed experts run on its grouped sm_100a "
                      "GEMMs when the model is on CUDA (any moe_dispatch), and on PyTorch on the CPU")
