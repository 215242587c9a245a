"""Import surface of the reference's ``models/mla_triton.py`` for code written
against it: ``HAS_TRITON``, ``mla_attention_reference`` and
``triton_mla_attention`` (reference ``models/mla_triton.py:28-67``, ``:303``).

This build has no Triton kernels.  MLA attention runs on its own sm_100a
kernels whenever the model runs on CUDA, whatever ``attn_impl`` says
(``models/_native_dispatch.py`` maps the reference's values onto them), so
``HAS_TRITON`` is always False and ``triton_mla_attention`` raises
``ImportError``.  ``mla_attention_reference`` is the fp32 CPU oracle the
kernel tests compare against: ``q_nope`` / ``q_pe`` ``[B, H, Sq, d]``,
latent context ``[B, Sk, R]`` / ``[B, Sk, dr]``, ``wkv_b_k`` / ``wkv_b_v``
``[H, d, R]``; returns ``[B, Sq, H, dv]``; ``is_causal`` masks keys after
``q_start + i`` for query ``i``.
"""
from ops.attention import mla_attention_reference

HAS_TRITON = False

__all__ = ["HAS_TRITON", "mla_attention_reference", "triton_mla_attention"]


def triton_mla_attention(*args, **kwargs):
    raise ImportError("triton kernels are not part of this build: MLA attention runs on its native sm_100a "
                      "kernels when the model is on CUDA (any attn_impl), and on PyTorch on the CPU")
