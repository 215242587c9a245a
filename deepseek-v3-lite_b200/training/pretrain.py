"""DeepSeek-V3-Lite pretraining: packed-token dataset, trainer and CLI.

Public surface and semantics match the reference (``training/pretrain.py``):

* ``TrainingConfig`` - same fields and defaults;
* ``PretrainDataset`` - packed LM windows from one ``torch.save``d 1-D token
  tensor or a directory of ``shard_*.bin`` files (mmap), windows may cross
  shard boundaries, ``len = (N - 1) // S``, item ``i`` is
  ``(chunk[:-1], chunk[1:])`` of ``chunk = tokens[i*S : i*S + S + 1]``;
* ``make_warmup_cosine_lambda`` - linear warmup, cosine to ``min_lr_ratio``
  over *optimizer* steps (``max_steps // grad_accum``), clamped after;
* ``Pretrainer`` - seeding, fp32 master model, optional MTP wrapper (only if
  ``mtp_depth > 0`` and ``mtp_weight > 0``), muP LR
  ``ref * sqrt(ref_params / params_incl_mtp)``, AdamW with two groups
  (dim >= 2 decayed), NaN guard with checkpoint rollback, auto-resume,
  aux-loss-free bias updates every ``bias_update_every`` optimizer steps;
* checkpoints in the reference's three-file format (``utils.checkpoint``).

What differs is the engine under ``train_step`` on CUDA: instead of autocast +
``torch.compile`` the step runs the hand-written sm_100a kernels through
``ops.engine.TrainEngine`` (fused MoE, MLA attention, fused LM-head
cross-entropy, fused AdamW over flat buffers), data-parallel gradient
reduce-scatter and expert parallelism when launched under ``torchrun``.  The
NaN guard reads a device flag instead of synchronising each micro-step.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import List, Dict, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
import yaml
from torch.optim import AdamW
from torch.optim.lr_scheduler import LambdaLR
from torch.utils.data import DataLoader, Dataset

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from models.mtp import MultiTokenPrediction  # noqa: E402
from models.transformer import Transformer, count_parameters  # noqa: E402
from utils.checkpoint import CheckpointManager  # noqa: E402
from utils.logging import get_logger, init_logging  # noqa: E402


def make_warmup_cosine_lambda(warmup_steps: int, total_steps: int, min_lr_ratio: float = 0.1):
    """LR multiplier: linear warmup, then cosine decay to ``min_lr_ratio``."""

    def factor(step: int) -> float:
        if step < warmup_steps:
            return step / max(1, warmup_steps)
        if step >= total_steps:
            return min_lr_ratio
        frac = (step - warmup_steps) / max(1, total_steps - warmup_steps)
        return min_lr_ratio + (1.0 - min_lr_ratio) * 0.5 * (1.0 + math.cos(math.pi * frac))

    return factor


@dataclass
class TrainingConfig:
    """All trainer knobs (defaults as in the reference)."""
    model_config: dict = field(default_factory=dict)
    data_path: str = "data/pretrain_data.bin"
    checkpoint_dir: str = "checkpoints/pretrain"
    vocab_size: int = 100018
    max_seq_len: int = 4096
    batch_size: int = 8
    gradient_accumulation_steps: int = 4
    max_steps: int = 20000
    warmup_steps: int = 2000
    lr: float = 2.2e-4
    min_lr_ratio: float = 0.1
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    max_grad_norm: float = 1.0
    mtp_weight: float = 0.0
    bias_update_speed: float = 0.001
    bias_update_every: int = 10
    grad_checkpoint: bool = True
    compile_model: bool = True
    save_every: int = 1000
    log_every: int = 100
    nan_guard: bool = False
    nan_guard_max_consecutive: int = 5
    mup_lr: bool = False
    mup_lr_reference: float = 6.0e-4
    mup_lr_reference_params: int = 757226496
    log_per_component_params: bool = True
    seed: int = 42
    # Expert-parallel group size (new; not in the reference, which is
    # single-device): 1 keeps every routed expert on every rank (plain data
    # parallelism), 0 spreads them over all ranks of the job.
    ep_size: int = 1
    # Receive-buffer cap of expert parallelism as a multiple of the mean load
    # (0: exact worst case, never overflows).
    ep_capacity_factor: float = 0.0
    # Shard routed-expert weights / gradients / optimizer state over the
    # expert-parallel ranks (needed when the experts do not fit on one GPU).
    ep_shard_experts: bool = False
    # Write checkpoints from a background thread after a host snapshot (new;
    # the reference saves synchronously).
    async_checkpoint: bool = False
    # Recompute each layer's forward in the fused engine's backward instead of
    # keeping its activations (new; `grad_checkpoint` keeps its reference
    # meaning for the eager module path).
    activation_recompute: bool = False


class PretrainDataset(Dataset):
    """Next-token training windows packed back to back over a token stream.

    The stream is either one ``torch.save``d 1-D token tensor or the
    concatenation, in file-name order, of a directory's ``shard_*.bin`` files
    (the reference's two layouts, ``training/pretrain.py:70-130``).  Window
    ``i`` is the ``max_seq_len + 1`` tokens starting at ``i * max_seq_len``,
    returned as ``(inputs, targets)`` shifted by one; a window may span shard
    files; the trailing partial window is dropped.

    Every file is memory-mapped once and becomes one segment of the stream;
    ``_ends`` holds each segment's exclusive end offset, so locating a token
    is one binary search and reading a window walks the segments it overlaps.
    """

    def __init__(self, data_path: str, max_seq_len: int, vocab_size: int):
        self.max_seq_len = int(max_seq_len)
        self.vocab_size = vocab_size
        root = Path(data_path)
        if not root.exists():
            raise FileNotFoundError(f"Pre-training data not found: {data_path}\n"
                                    "Build token shards first (data/prepare_data.py or data/build_small_shard.py).")
        self.layout = "sharded" if root.is_dir() else "single"
        files = sorted(root.glob("shard_*.bin")) if root.is_dir() else [root]
        if not files:
            raise FileNotFoundError(f"{data_path} is a directory without shard_*.bin token files")
        self.shard_paths = [str(f) for f in files]
        self._segments = [torch.load(f, map_location="cpu", weights_only=True, mmap=True).reshape(-1) for f in files]
        self._ends = np.cumsum([seg.numel() for seg in self._segments], dtype=np.int64)
        self._total_tokens = int(self._ends[-1])

    def _locate(self, global_idx: int) -> Tuple[int, int]:
        """``(segment, offset)`` of stream position ``global_idx``; ``IndexError`` outside the stream."""
        if not 0 <= global_idx < self._total_tokens:
            raise IndexError(f"global_idx {global_idx} out of range [0, {self._total_tokens})")
        seg = int(np.searchsorted(self._ends, global_idx, side="right"))
        return seg, global_idx - (int(self._ends[seg - 1]) if seg else 0)

    def _read(self, begin: int, count: int) -> torch.Tensor:
        seg, off = self._locate(begin)
        pieces = []
        while count > 0:
            piece = self._segments[seg][off:off + count]
            pieces.append(piece)
            count -= piece.numel()
            seg, off = seg + 1, 0
        return torch.cat(pieces) if len(pieces) > 1 else pieces[0].clone()

    def __len__(self) -> int:
        return max(0, (self._total_tokens - 1) // self.max_seq_len)

    def __getitem__(self, idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        window = self._read(idx * self.max_seq_len, self.max_seq_len + 1)
        return window[:-1], window[1:]


class _LazyMetric:
    """A diagnostic computed only when read (``float()`` / ``.item()``), so the
    per-micro-step hot path does not pay for it."""

    def __init__(self, fn):
        self._fn = fn
        self._v = None

    def _get(self) -> torch.Tensor:
        if self._v is None:
            self._v = self._fn()
        return self._v

    def item(self) -> float:
        return float(self._get().item())

    def __float__(self) -> float:
        return self.item()


def _unique_params(module: nn.Module):
    seen, out = set(), []
    for p in module.parameters():
        if id(p) not in seen:
            seen.add(id(p))
            out.append(p)
    return out


class Pretrainer:
    """Resumable pretraining loop (single process, or one rank of a torchrun job)."""

    def __init__(self, config: TrainingConfig):
        self.config = config
        torch.manual_seed(config.seed)
        self.device = self._pick_device()
        if self.device.type == "cuda":
            torch.backends.cuda.matmul.allow_tf32 = True
            torch.backends.cudnn.allow_tf32 = True
            torch.set_float32_matmul_precision("high")
        else:
            print("[warn] CUDA not available - running on CPU (smoke-testing only).")
        init_logging(config.log_every, seq_len=config.max_seq_len, batch_size=config.batch_size)
        self.logger = get_logger()

        self._log("Initialising model...")
        model_cfg = config.model_config.get("model", config.model_config)
        # built on the training device directly: a 14B-parameter model in fp32
        # would otherwise take 55 GB of host memory per rank
        with torch.device(self.device):
            raw = Transformer(config.model_config, use_checkpoint=config.grad_checkpoint)
        total, trainable = count_parameters(raw)
        self._log(f"Parameters: {total:,} total / {trainable:,} trainable")
        if config.log_per_component_params:
            self._log_per_component_params(raw)
        self.mtp_wrapper: Optional[MultiTokenPrediction] = None
        training_model: nn.Module = raw
        if model_cfg.get("mtp_depth", 0) > 0 and config.mtp_weight > 0.0:
            with torch.device(self.device):
                self.mtp_wrapper = MultiTokenPrediction(config.model_config, raw)
            total, trainable = count_parameters(self.mtp_wrapper)
            self._log(f"MTP enabled (depth={self.mtp_wrapper.depth}, weight={config.mtp_weight}): "
                      f"{total:,} total / {trainable:,} trainable")
            training_model = self.mtp_wrapper
        # No tracing compiler: compile_model is accepted for config compatibility;
        # the CUDA step runs hand-written kernels captured in CUDA graphs instead.
        self.model = training_model
        self.raw_model: Transformer = raw

        if config.mup_lr:
            new_lr = config.mup_lr_reference * (config.mup_lr_reference_params / total) ** 0.5
            self._log(f"muP LR scaling: {config.lr:.2e} -> {new_lr:.2e} "
                      f"(ref {config.mup_lr_reference:.2e} @ {config.mup_lr_reference_params:,} params)")
            config.lr = new_lr

        params = _unique_params(self.model)
        groups = [
            {"params": [p for p in params if p.dim() >= 2], "weight_decay": config.weight_decay},
            {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0},
        ]
        self.engine = None
        if self.device.type == "cuda":
            self._memory_hint(config)
            from ops.engine import TrainEngine
            self.engine = TrainEngine(self.raw_model, self.mtp_wrapper, config, groups)
            self.optimizer = self.engine.optimizer
        else:
            self.optimizer = AdamW(groups, lr=config.lr, betas=(config.beta1, config.beta2), foreach=False)
        horizon = max(1, config.max_steps // config.gradient_accumulation_steps)
        self.scheduler = LambdaLR(self.optimizer, make_warmup_cosine_lambda(config.warmup_steps, horizon,
                                                                            config.min_lr_ratio))
        self.amp_dtype = torch.bfloat16
        self.ckpt_manager = CheckpointManager(config.checkpoint_dir)
        self._opt_steps = 0

    # --------------------------------------------------------------- helpers
    def _memory_hint(self, config: TrainingConfig) -> None:
        """Warn (never fail) when the estimated per-rank training state does
        not fit the device, naming expert sharding when that would fix it."""
        try:
            from utils.memory import expert_sharding_hint
            dist_on = torch.distributed.is_available() and torch.distributed.is_initialized()
            world = torch.distributed.get_world_size() if dist_on else 1
            device_gb = torch.cuda.get_device_properties(self.device).total_memory / 1024 ** 3
            hint = expert_sharding_hint(self.raw_model, config.max_seq_len, config.batch_size, world,
                                        int(config.ep_size), bool(config.ep_shard_experts), device_gb)
            if hint:
                self._log(f"[warn] {hint}")
        except Exception as exc:  # an estimate must never stop training
            self._log(f"[warn] memory estimate skipped: {exc}")

    @staticmethod
    def _pick_device() -> torch.device:
        if not torch.cuda.is_available():
            return torch.device("cpu")
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        return torch.device("cuda", local)

    @staticmethod
    def _log(msg: str) -> None:
        if int(os.environ.get("RANK", "0")) == 0:
            print(msg)

    def _amp_context(self):
        return torch.autocast(self.device.type, dtype=self.amp_dtype)

    def _update_moe_bias(self) -> None:
        dp = getattr(self.engine, "dp", None) if self.engine is not None else None
        for moe in self.raw_model.moe_layers():
            if dp is not None and moe.expert_counts() is not None:
                # every rank applies the same update from the global counts
                moe.gate.update_bias(dp.global_counts(moe.expert_counts()), speed=self.config.bias_update_speed)
            else:
                moe.update_gate_bias(speed=self.config.bias_update_speed)

    def expert_load_histograms(self) -> Dict[int, List[int]]:
        """Routed rows per expert of each MoE layer in the last micro-batch
        (this rank's tokens; a by-product of the router kernel)."""
        out = {}
        for i, layer in enumerate(self.raw_model.layers):
            ffn = layer.ffn
            if hasattr(ffn, "expert_counts") and ffn.expert_counts() is not None:
                out[i] = [int(c) for c in ffn.expert_counts().tolist()]
        return out

    def step_diagnostics(self) -> Dict[str, float]:
        """Logged next to the loss: global gradient norm, worst per-layer
        expert load (max / mean routed rows) and, under expert parallelism,
        the bytes of token rows this rank sent to other ranks per MoE layer
        and direction in the last micro-batch."""
        d: Dict[str, float] = {}
        eng = self.engine
        if eng is not None:
            d["grad_norm"] = float(eng.optimizer.grad_norm)
        worst = 0.0
        for counts in self.expert_load_histograms().values():
            mean = sum(counts) / max(1, len(counts))
            if mean > 0:
                worst = max(worst, max(counts) / mean)
        if worst:
            d["expert_load_max_over_mean"] = worst
        if eng is not None and getattr(eng, "ep", None) is not None:
            ep = eng.ep
            counts = next(iter(self.expert_load_histograms().values()), None)
            if counts is not None:
                remote = sum(counts) - sum(counts[ep.lo:ep.hi])
                d["ep_bytes_sent_per_layer"] = float(remote * ep.D * 2)
        return d

    def _moe_balance_metric(self) -> torch.Tensor:
        """Sum of per-layer balance metrics (device tensor; read lazily)."""
        vals = [moe.get_load_balance_loss() for moe in self.raw_model.moe_layers()]
        return torch.stack(vals).sum() if vals else torch.tensor(0.0, device=self.device)

    def _log_per_component_params(self, model: nn.Module) -> None:
        buckets: Dict[str, int] = {}
        seen = set()
        for name, p in model.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            if "embed" in name:
                key = "embedding"
            elif "head" in name:
                key = "lm_head"
            elif ".attn." in name and any(s in name for s in ("wq", "wkv_a", "wkv_b", "wo", "q_norm", "kv_norm")):
                key = "mla_attn"
            elif "attn_norm" in name or "ffn_norm" in name or name.endswith(".norm.weight") or name == "norm.weight":
                key = "rmsnorm"
            elif "shared_experts" in name:
                key = "moe_shared_experts"
            elif ".experts." in name:
                key = "moe_routed_experts"
            elif ".ffn.w" in name:
                key = "dense_swiglu"
            elif ".gate." in name:
                key = "moe_gate"
            else:
                key = "other"
            buckets[key] = buckets.get(key, 0) + p.numel()
        total = sum(buckets.values())
        self._log("  Per-component parameter breakdown:")
        for key, n in sorted(buckets.items(), key=lambda kv: -kv[1]):
            self._log(f"    {key:25s}: {n:>12,}  ({100.0 * n / max(total, 1):5.2f}%)")
        self._log(f"    {'TOTAL':25s}: {total:>12,}  ({total / 1e6:.2f} M)")

    # ------------------------------------------------------------ train step
    def train_step(self, tokens: torch.Tensor, targets: torch.Tensor, micro_step: int) -> Optional[Dict]:
        """One micro-batch; steps the optimizer at the accumulation boundary.

        Returns ``{"loss", "mtp_loss", "balance_loss"}`` (device tensors) or
        ``None`` when the NaN guard skipped the micro-batch.
        """
        accum = self.config.gradient_accumulation_steps
        boundary = (micro_step + 1) % accum == 0
        tokens = tokens.long() if tokens.dtype != torch.long else tokens
        targets = targets.long() if targets.dtype != torch.long else targets
        if self.engine is not None:
            return self._engine_step(tokens, targets, boundary)
        with self._amp_context():
            if self.mtp_wrapper is not None:
                main_logits, pairs = self.model(tokens)
                total, main, mtp = self.mtp_wrapper.compute_loss(main_logits, targets, pairs)
                mtp_val = mtp.detach() if pairs else None
            else:
                logits = self.model(tokens, start_pos=0, use_cache=False)
                main = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1),
                                                         ignore_index=-100)
                total, mtp_val = main, None
            loss = total / accum
            balance = self._moe_balance_metric()
        if self.config.nan_guard and not bool(torch.isfinite(loss).all()):
            self._log(f"[nan-guard] NaN/Inf at micro_step={micro_step}, opt_steps={self._opt_steps}. Skipping backward.")
            self.optimizer.zero_grad(set_to_none=True)
            return None
        loss.backward()
        if boundary:
            nn.utils.clip_grad_norm_(self.model.parameters(), self.config.max_grad_norm)
            self.optimizer.step()
            self.scheduler.step()
            self.optimizer.zero_grad(set_to_none=True)
            self._after_opt_step()
        return {"loss": main.detach(), "mtp_loss": mtp_val, "balance_loss": balance}

    def _after_opt_step(self) -> None:
        self._opt_steps += 1
        if self._opt_steps % self.config.bias_update_every == 0:
            self._update_moe_bias()

    def _engine_step(self, tokens, targets, boundary: bool) -> Optional[Dict]:
        eng = self.engine
        out = eng.forward_backward(tokens, targets, loss_scale=1.0 / self.config.gradient_accumulation_steps)
        out["balance_loss"] = _LazyMetric(self._moe_balance_metric)
        if self.config.nan_guard and not eng.last_loss_finite():
            self._log(f"[nan-guard] NaN/Inf loss, opt_steps={self._opt_steps}. Dropping accumulated gradients.")
            eng.zero_grad()
            return None
        if boundary:
            eng.clip_and_step(self.config.max_grad_norm)
            self.scheduler.step()
            eng.zero_grad()
            self._after_opt_step()
        return out

    # ----------------------------------------------------------- checkpoints
    def save_checkpoint(self, step: int, tag: str = "") -> None:
        """Write model (+MTP) weights, optimizer state and metadata for ``step``."""
        sharded = self.engine is not None and getattr(self.engine, "shard_experts", False)
        if self.engine is not None:
            self.engine.sync_to_modules()
        state = self.raw_model.state_dict()
        if getattr(self.raw_model, "weight_tying", False):
            state.pop("head.weight", None)
        if self.mtp_wrapper is not None:
            state.update({f"mtp.{k}": v for k, v in self.mtp_wrapper.state_dict().items()
                          if k.startswith("mtp_modules.")})
        meta = {"scheduler": self.scheduler.state_dict(), "opt_steps": self._opt_steps,
                "tag": tag or f"step_{step}", "config": asdict(self.config),
                "has_mtp": self.mtp_wrapper is not None}
        opt_state = self.engine.optimizer_state_for_checkpoint() if self.engine is not None else None
        if sharded:
            # routed experts: one file per owner, written before rank 0's
            # metadata makes the step visible
            eng = self.engine
            state = {k: v for k, v in state.items() if ".experts." not in k}
            expert_ids = {id(p) for n, p in self.raw_model.named_parameters() if ".experts." in n}
            order = [p for g in self.optimizer.param_groups for p in g["params"]]
            for i, p in enumerate(order):
                if id(p) in expert_ids:
                    opt_state["state"].pop(i, None)
            meta["expert_shards"] = eng.world_size
            self.ckpt_manager.save_expert_shard(step, eng.rank, eng.world_size, eng.expert_shard_state())
            torch.distributed.barrier(group=eng.dp.group)
        if int(os.environ.get("RANK", "0")) == 0:
            self.ckpt_manager.save(self.raw_model, self.optimizer, step, extra_meta=meta, state_dict=state,
                                   optimizer_state=opt_state, background=self.config.async_checkpoint)
        self._log(f"Checkpoint {'queued' if self.config.async_checkpoint else 'saved'} at step {step}")

    def load_checkpoint(self, step: int) -> int:
        """Restore ``step`` (weights, optimizer, MTP, scheduler, opt-step count)."""
        from safetensors.torch import load_file
        sharded = self.engine is not None and getattr(self.engine, "shard_experts", False)
        meta = self.ckpt_manager.load(self.raw_model, step, device=str(self.device), optimizer=self.optimizer,
                                      strict=False, merge_expert_shards=not sharded)
        if sharded:
            eng = self.engine
            saved = int(meta.get("expert_shards", 0) or 0)
            if saved != eng.world_size:
                raise RuntimeError(f"step {step} holds {saved} expert shards; resume with {saved} ranks "
                                   f"(or load it unsharded, which merges the shards' weights)")
            eng.load_expert_shard_state(self.ckpt_manager.load_expert_shard(step, eng.rank, saved,
                                                                            device=str(self.device)))
        if self.mtp_wrapper is not None and meta.get("has_mtp", False):
            wpath = self.ckpt_manager.save_dir / f"model_step_{step}.safetensors"
            if wpath.exists():
                mtp_state = {k[len("mtp."):]: v for k, v in load_file(str(wpath), device=str(self.device)).items()
                             if k.startswith("mtp.")}
                if mtp_state:
                    self.mtp_wrapper.load_state_dict(mtp_state, strict=False)
                    self._log(f"MTP weights restored ({len(mtp_state)} keys)")
        if "scheduler" in meta:
            self.scheduler.load_state_dict(meta["scheduler"])
        if "opt_steps" in meta:
            self._opt_steps = meta["opt_steps"]
        if self.engine is not None:
            self.engine.sync_from_modules()
        resumed = meta.get("step", step)
        self._log(f"Resumed from step {resumed}")
        return resumed

    def _find_latest_checkpoint(self) -> Optional[int]:
        return self.ckpt_manager.latest_step()

    # ------------------------------------------------------------------ loop
    def _make_loader(self) -> DataLoader:
        ds = PretrainDataset(self.config.data_path, self.config.max_seq_len, self.config.vocab_size)
        gen = torch.Generator().manual_seed(self.config.seed)
        sampler = None
        if self.engine is not None and self.engine.world_size > 1:
            from torch.utils.data.distributed import DistributedSampler
            sampler = DistributedSampler(ds, num_replicas=self.engine.world_size, rank=self.engine.rank,
                                         shuffle=True, seed=self.config.seed, drop_last=True)
        workers = min(8, os.cpu_count() or 1)
        return DataLoader(ds, batch_size=self.config.batch_size, shuffle=sampler is None, sampler=sampler,
                          generator=gen if sampler is None else None, num_workers=workers,
                          pin_memory=self.device.type == "cuda", persistent_workers=workers > 0,
                          prefetch_factor=8 if workers > 0 else None, drop_last=True)

    def train(self) -> None:
        """Train until ``max_steps`` micro-steps, resuming from the latest checkpoint."""
        loader = self._make_loader()
        step = 0
        latest = self._find_latest_checkpoint()
        if latest is not None:
            try:
                step = self.load_checkpoint(latest)
            except Exception as exc:  # corrupted or incompatible checkpoint
                self._log(f"[warn] Could not load checkpoint: {exc}")
        self._log(f"Training from step {step} to {self.config.max_steps}")
        self.raw_model.train()
        try:
            step = self._train_loop(loader, step)
            self.save_checkpoint(step, tag="final")
        except BaseException:
            # a background checkpoint write that failed must not go unseen
            # behind the training error
            try:
                self.ckpt_manager.wait()
            except Exception as exc:
                self._log(f"[warn] background checkpoint write failed: {exc}")
            raise
        self.ckpt_manager.wait()
        self._log("Training complete.")

    def _train_loop(self, loader, step: int) -> int:
        streak = 0
        while step < self.config.max_steps:
            for tokens, targets in loader:
                if step >= self.config.max_steps:
                    break
                tokens = tokens.to(self.device, non_blocking=True)
                targets = targets.to(self.device, non_blocking=True)
                metrics = self.train_step(tokens, targets, step)
                if metrics is None:
                    streak += 1
                    if streak >= self.config.nan_guard_max_consecutive:
                        latest = self._find_latest_checkpoint()
                        if latest is None:
                            self._log("[nan-guard] No checkpoint to restore from. Aborting.")
                            raise RuntimeError("NaN/Inf with no checkpoint to restore from")
                        self._log(f"[nan-guard] {streak} consecutive NaN/Inf - restoring checkpoint step {latest}.")
                        step = self.load_checkpoint(latest)
                        streak = 0
                    continue
                streak = 0
                extras = None
                if step % self.config.log_every == 0:
                    extras = {"balance_loss": float(metrics["balance_loss"])}
                    if metrics.get("mtp_loss") is not None:
                        extras["mtp_loss"] = float(metrics["mtp_loss"])
                    extras.update(self.step_diagnostics())
                # the loss stays on the device; the logger reads it once per interval
                self.logger.log(step, metrics["loss"], lr=self.scheduler.get_last_lr()[0], metrics=extras)
                if step % self.config.save_every == 0 and step > 0:
                    self.save_checkpoint(step)
                step += 1
        return step


def config_from_yaml(yaml_cfg: dict, data_path: Optional[str] = None, checkpoint_dir: Optional[str] = None,
                     no_checkpoint: bool = False, no_compile: bool = False) -> TrainingConfig:
    """Map a YAML dict (``model``/``training``/``data``) onto ``TrainingConfig``."""
    t, d = yaml_cfg.get("training", {}), yaml_cfg.get("data", {})
    m = yaml_cfg.get("model", yaml_cfg)
    return TrainingConfig(
        model_config=yaml_cfg,
        data_path=data_path or d.get("train_data_path", "data/pretrain_data.bin"),
        checkpoint_dir=checkpoint_dir or t.get("save_dir", "checkpoints/pretrain"),
        max_seq_len=m.get("max_seq_len", 4096),
        vocab_size=m.get("vocab_size", 100018),
        batch_size=t.get("micro_batch_size", 8),
        gradient_accumulation_steps=t.get("gradient_accumulation_steps", 4),
        max_steps=t.get("total_steps", 20000),
        warmup_steps=t.get("warmup_steps", 2000),
        lr=t.get("lr", 2.2e-4),
        min_lr_ratio=t.get("min_lr_ratio", 0.1),
        weight_decay=t.get("weight_decay", 0.1),
        max_grad_norm=t.get("grad_clip", 1.0),
        grad_checkpoint=t.get("grad_checkpoint", True) and not no_checkpoint,
        compile_model=t.get("compile", True) and not no_compile,
        mtp_weight=t.get("mtp_loss_weight", 0.0),
        bias_update_speed=t.get("bias_update_speed", 0.001),
        bias_update_every=t.get("bias_update_every", 10),
        save_every=t.get("save_interval", 1000),
        log_every=t.get("log_interval", 100),
        nan_guard=t.get("nan_guard", False),
        nan_guard_max_consecutive=t.get("nan_guard_max_consecutive", 5),
        mup_lr=t.get("mup_lr", False),
        mup_lr_reference=t.get("mup_lr_reference", 6.0e-4),
        mup_lr_reference_params=t.get("mup_lr_reference_params", 757226496),
        log_per_component_params=t.get("log_per_component_params", True),
        seed=t.get("seed", 42),
        ep_size=int(yaml_cfg.get("parallel", {}).get("ep_size", 1)),
        ep_capacity_factor=float(yaml_cfg.get("parallel", {}).get("ep_capacity_factor", 0.0)),
        ep_shard_experts=bool(yaml_cfg.get("parallel", {}).get("shard_experts", False)),
        async_checkpoint=bool(t.get("async_checkpoint", False)),
        activation_recompute=bool(t.get("activation_recompute", False)),
    )


def main() -> None:
    """CLI: ``python training/pretrain.py --config cfg.yaml [...]`` (or under torchrun)."""
    ap = argparse.ArgumentParser(description="DeepSeek-V3-Lite pre-training on B200")
    ap.add_argument("--config", type=str, default=str(Path(__file__).resolve().parent.parent / "configs" / "pretrain_412m.yaml"))
    ap.add_argument("--data-path", type=str, default=None)
    ap.add_argument("--checkpoint-dir", type=str, default=None)
    ap.add_argument("--resume", type=str, default=None, help="Checkpoint step number to resume from")
    ap.add_argument("--no-checkpoint", action="store_true", help="Disable activation checkpointing")
    ap.add_argument("--no-compile", action="store_true", help="Accepted for compatibility (no compiler is used)")
    args = ap.parse_args()
    with open(args.config) as f:
        yaml_cfg = yaml.safe_load(f)
    cfg = config_from_yaml(yaml_cfg, args.data_path, args.checkpoint_dir, args.no_checkpoint, args.no_compile)
    trainer = Pretrainer(cfg)
    if args.resume is not None:
        trainer.load_checkpoint(int(args.resume))
    trainer.train()


if __name__ == "__main__":
    main()
