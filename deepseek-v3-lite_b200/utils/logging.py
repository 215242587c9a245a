"""Training-progress logger.

Interface kept from the reference (``utils/logging.py:7-65``): the
``TrainingLogger(log_interval, seq_len, batch_size)`` constructor, ``log(step,
loss, metrics, lr)``, the process-wide ``init_logging`` / ``get_logger``, the
line ``step=... | loss=... | ppl=... | lr=... | tps=... | k=v`` and the
Weights & Biases keys ``train/<name>`` (enabled by ``WANDB_PROJECT``,
``WANDB_RUN_NAME`` names the run).

Design: the loss may be handed over as a device tensor every micro-step; the
logger keeps a running device-side sum and reads it once per interval, so the
training loop never synchronises on the loss between emitted lines.  The
interval's throughput is counted as ``log_interval * seq_len * batch_size``
tokens over the monotonic wall time between two emitted lines (device-timed
throughput, CUDA events and max over ranks, is what ``bench.py`` reports).
"""
from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, Optional, Union

import torch

Number = Union[float, int, torch.Tensor]


@dataclass
class _Interval:
    """Loss samples since the last emitted line: host floats and device tensors kept apart."""

    opened: float = field(default_factory=time.perf_counter)
    count: int = 0
    host_total: float = 0.0
    device_total: Optional[torch.Tensor] = None

    def add(self, loss: Number) -> None:
        self.count += 1
        if isinstance(loss, torch.Tensor) and loss.device.type != "cpu":
            v = loss.detach().reshape(()).float()
            self.device_total = v.clone() if self.device_total is None else self.device_total.add_(v)
        else:
            self.host_total += float(loss)

    def mean(self) -> float:
        total = self.host_total
        if self.device_total is not None:
            total += float(self.device_total)        # the interval's only device read
        return total / max(1, self.count)


def format_line(step: int, loss: float, lr: float, tokens_per_s: float, extras: Dict[str, float]) -> str:
    """One progress line in the reference's format."""
    head = [f"step={step:>7}", f"loss={loss:.4f}", f"ppl={math.exp(min(loss, 700.0)):.2f}",
            f"lr={lr:.2e}", f"tps={tokens_per_s:,.0f}"]
    return " | ".join(head + [f"{k}={float(v):.4f}" for k, v in extras.items()])


def _wandb_sink() -> Optional[Callable[[Dict[str, float], int], None]]:
    project = os.environ.get("WANDB_PROJECT")
    if not project:
        return None
    try:
        import wandb
        wandb.init(project=project, name=os.environ.get("WANDB_RUN_NAME"), reinit=True)
    except Exception as exc:  # not installed, offline, or refused
        print(f"[logging] wandb disabled: {exc}")
        return None
    return lambda payload, step: wandb.log(payload, step=step)


class TrainingLogger:
    """Averages the loss over ``log_interval`` steps and emits one line per interval."""

    def __init__(self, log_interval: int = 10, seq_len: int = 1024, batch_size: int = 1):
        self.log_interval = max(1, int(log_interval))
        self.seq_len = seq_len
        self.batch_size = batch_size
        self._interval = _Interval()
        self._sink = _wandb_sink()
        self.last_line: Optional[str] = None

    @property
    def tokens_per_interval(self) -> int:
        return self.log_interval * self.seq_len * self.batch_size

    def log(self, step: int, loss: Number, metrics: Optional[Dict[str, float]] = None, lr: float = 0.0) -> None:
        """Add ``loss`` (a float or a device scalar) to the interval; emit when ``step`` is a multiple of it."""
        self._interval.add(loss)
        if step % self.log_interval:
            return
        closing, self._interval = self._interval, _Interval()
        mean = closing.mean()
        tps = self.tokens_per_interval / max(self._interval.opened - closing.opened, 1e-6)
        extras = dict(metrics or {})
        self.last_line = format_line(step, mean, lr, tps, extras)
        print(self.last_line)
        if self._sink is not None:
            payload = {"train/loss": mean, "train/ppl": math.exp(min(mean, 700.0)), "train/lr": lr,
                       "train/tokens_per_sec": tps}
            payload.update({f"train/{k}": float(v) for k, v in extras.items()})
            self._sink(payload, step)


_logger: Optional[TrainingLogger] = None


def init_logging(log_interval: int = 10, seq_len: int = 1024, batch_size: int = 1) -> None:
    """Create the process-wide logger."""
    global _logger
    _logger = TrainingLogger(log_interval, seq_len, batch_size)


def get_logger() -> TrainingLogger:
    """The process-wide logger (created with defaults on first use)."""
    global _logger
    if _logger is None:
        _logger = TrainingLogger()
    return _logger
