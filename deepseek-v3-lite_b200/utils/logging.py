"""Training-progress logger.

Line format and optional Weights & Biases forwarding follow the reference
(``utils/logging.py:7-65``): ``step=... | loss=... | ppl=... | lr=... | tps=...``
followed by ``k=v`` extras; wandb keys are ``train/<name>`` and wandb is
enabled by ``WANDB_PROJECT`` (``WANDB_RUN_NAME`` names the run).

``tps`` here is *wall-clock* throughput between two emitted lines, counted as
``log_interval * seq_len * batch_size`` tokens.  Device-timed throughput (CUDA
events, max over ranks) is reported by ``utils.timing`` and ``bench.py``.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, Optional


class TrainingLogger:
    """Average the loss over an interval and print one summary line per interval."""

    def __init__(self, log_interval: int = 10, seq_len: int = 1024, batch_size: int = 1):
        self.log_interval = max(1, int(log_interval))
        self.seq_len = seq_len
        self.batch_size = batch_size
        self._start = time.time()
        self._step_start = time.time()
        self._loss_window: list = []
        self._wandb = None
        project = os.environ.get("WANDB_PROJECT")
        if project:
            try:
                import wandb
                wandb.init(project=project, name=os.environ.get("WANDB_RUN_NAME"), reinit=True)
                self._wandb = wandb
            except Exception as exc:  # wandb missing or offline
                print(f"[logging] wandb disabled: {exc}")

    def log(self, step: int, loss: float, metrics: Optional[Dict[str, float]] = None, lr: float = 0.0) -> None:
        """Record ``loss`` for ``step``; print a line when ``step`` hits the interval."""
        self._loss_window.append(float(loss))
        if step % self.log_interval != 0:
            return
        avg = sum(self._loss_window) / len(self._loss_window)
        elapsed = max(time.time() - self._step_start, 1e-6)
        tps = self.log_interval * self.seq_len * self.batch_size / elapsed
        ppl = math.exp(min(avg, 700.0))
        parts = [f"step={step:>7}", f"loss={avg:.4f}", f"ppl={ppl:.2f}", f"lr={lr:.2e}", f"tps={tps:,.0f}"]
        parts += [f"{k}={v:.4f}" for k, v in (metrics or {}).items()]
        print(" | ".join(parts))
        if self._wandb is not None:
            payload = {"train/loss": avg, "train/ppl": ppl, "train/lr": lr, "train/tokens_per_sec": tps}
            payload.update({f"train/{k}": v for k, v in (metrics or {}).items()})
            self._wandb.log(payload, step=step)
        self._loss_window = []
        self._step_start = time.time()


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
