"""Loader for the in-tree sm_100a extension ``ops/_dsv3_C*.so``.

CUDA code paths call ``native()``; if the library is missing they raise
instead of falling back to another implementation, so a GPU run can never
silently measure something other than these kernels.
"""
from __future__ import annotations

import importlib

import torch  # noqa: F401  (loads libc10 / libtorch before the extension)

_mod = None
_err = None

# Kernels launched per entry point (entries not listed launch one kernel).
_LAUNCHES_PER_CALL = {"ce_reduce": 2, "flash_bwd": 2, "flash_bwd_wide": 3, "latent_decode": 2, "grad_sqsum": 3,
                      "status_read": 0, "status_reset": 0, "moe_norm_bwd_smem": 0,
                      "decode_tc": 0, "gemm_pairs": 0}
_counting = [False, 0]


class _CountingModule:
    """Forwards to the extension; while counting is on, tallies kernel launches."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        w = self._cache.get(name)
        if w is None:
            n = _LAUNCHES_PER_CALL.get(name, 1)

            def w(*a, **k):
                if _counting[0]:
                    _counting[1] += n
                return fn(*a, **k)
            self._cache[name] = w
        return w


def count_launches(enable: bool) -> int:
    """Start (``True``) or stop (``False``) counting; returns the count so far."""
    n = _counting[1]
    _counting[0] = enable
    if enable:
        _counting[1] = 0
    return n


def add_launches(n: int) -> None:
    """Account for ``n`` kernels launched outside the wrapper (a CUDA-graph replay)."""
    if _counting[0]:
        _counting[1] += n


class launch_scope:
    """Counts the kernel launches issued inside the ``with`` block (e.g. the
    nodes a CUDA-graph capture records) without disturbing an outer count."""

    def __enter__(self):
        self._outer = (_counting[0], _counting[1])
        _counting[0], _counting[1] = True, 0
        self.count = 0
        return self

    def __exit__(self, *exc):
        self.count = _counting[1]
        _counting[0], _counting[1] = self._outer
        return False


def native():
    """The compiled kernel module; raises ``RuntimeError`` if it is not built."""
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        _mod = _CountingModule(importlib.import_module("ops._dsv3_C"))
    except ImportError as exc:  # not built, or built for another interpreter
        _err = exc
        raise RuntimeError(
            "The sm_100a kernel library ops/_dsv3_C is not built. Run "
            "`python setup.py build_ext --inplace` in deepseek-v3-lite_b200/ "
            f"(or __graft_entry__.build()). Import error: {exc}") from exc
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def check_status() -> None:
    """Raise if any kernel recorded a bounded-wait timeout or a bounds failure."""
    code = native().status_read()
    if code:
        names = {1: "TMA stage wait", 2: "free-stage wait", 3: "TMEM hand-off wait", 4: "peer flag wait",
                 5: "index bounds check"}
        native().status_reset()
        raise RuntimeError(f"sm_100a kernel reported error {code} ({names.get(code, 'unknown')})")
