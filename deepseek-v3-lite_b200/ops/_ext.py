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


def native():
    """The compiled kernel module; raises ``RuntimeError`` if it is not built."""
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        _mod = importlib.import_module("ops._dsv3_C")
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
