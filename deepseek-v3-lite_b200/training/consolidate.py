"""Turn a checkpoint written with sharded routed experts into a plain one.

Training with ``parallel.shard_experts`` writes each rank's routed experts
(weights and AdamW moments) to its own ``experts_step_N_rankRofW`` file and
leaves them out of the model and optimizer files.  This tool merges them
back: the result is the usual three-file checkpoint (``model_step_N``,
``optim_step_N``, ``meta_step_N``) with every expert weight under its
state-dict name and every expert's moments in the optimizer state at the
index a single-process trainer gives that parameter (decayed parameters
first, then undecayed, each in module order, as
``training/pretrain.py:Pretrainer`` groups them; the reference's
``training/pretrain.py`` uses the same order).  Such a checkpoint resumes in
an unsharded run, or in a sharded run of any size after it is sharded again
by training, and loads in the reference's own trainer.

Runs on the CPU; the model is instantiated on the ``meta`` device only to
learn parameter names, shapes and order, so a 14B configuration needs no
memory for its weights beyond the tensors being merged.

``python -m training.consolidate --checkpoint-dir DIR [--step N] --out-dir OUT``
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path
from typing import Dict, Optional

import torch
from safetensors.torch import load_file

from utils.checkpoint import CheckpointManager

_AVG, _SQ = "exp_avg.", "exp_avg_sq."


def optimizer_index(model_config: dict, has_mtp: bool) -> Dict[str, int]:
    """State-dict name of every parameter of the main model (and, with MTP,
    ``mtp.``-prefixed MTP parameters) -> its index in the trainer's
    optimizer state."""
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    with torch.device("meta"):
        raw = Transformer(model_config)
        model = MultiTokenPrediction(model_config, raw) if has_mtp else raw
    named = list(model.named_parameters())
    order = [n for n, p in named if p.dim() >= 2] + [n for n, p in named if p.dim() < 2]
    index = {}
    for i, n in enumerate(order):
        if has_mtp and n.startswith("main_model."):
            n = n[len("main_model."):]
        elif has_mtp:
            n = "mtp." + n
        index[n] = i
    return index


def consolidate(save_dir: str, out_dir: str, step: Optional[int] = None) -> int:
    """Write the merged checkpoint of ``step`` (default: the latest) into
    ``out_dir``; returns the step."""
    src = CheckpointManager(save_dir)
    step = src.latest_step() if step is None else step
    if step is None:
        raise FileNotFoundError(f"no complete checkpoint in {save_dir}")
    meta = src._meta(step)
    shards = int(meta.get("expert_shards", 0) or 0)
    if shards <= 0:
        raise ValueError(f"step {step} in {save_dir} has no expert shards; it is already a plain checkpoint")
    model_config = meta["config"]["model_config"]
    has_mtp = bool(meta.get("has_mtp", False))
    index = optimizer_index(model_config, has_mtp)

    weights = load_file(str(src._path(0, step)), device="cpu")
    optim = torch.load(src._path(1, step), map_location="cpu", weights_only=True)
    state = optim["state"]
    some = next(iter(state.values()), None)
    step_value = some["step"].clone() if some is not None else torch.tensor(float(meta.get("opt_steps", 0)))
    merged = set()
    for r in range(shards):
        for k, v in src.load_expert_shard(step, r, shards).items():
            if k.startswith(_SQ) or k.startswith(_AVG):
                slot, name = ("exp_avg_sq", k[len(_SQ):]) if k.startswith(_SQ) else ("exp_avg", k[len(_AVG):])
                if name not in index:
                    raise KeyError(f"shard {r} holds moments of unknown parameter {name}")
                state.setdefault(index[name], {"step": step_value.clone()})[slot] = v
            else:
                if k not in index:
                    raise KeyError(f"shard {r} holds unknown parameter {k}")
                weights[k] = v
                merged.add(k)
    experts = {n for n in index if ".experts." in n}
    missing = sorted(experts - merged)
    incomplete = sorted(n for n in experts if not {"exp_avg", "exp_avg_sq"} <= set(state.get(index[n], {})))
    if missing or incomplete:
        raise RuntimeError(f"expert shards of step {step} are incomplete: {len(missing)} weights missing "
                           f"({missing[:3]}), {len(incomplete)} without moments ({incomplete[:3]})")
    out = CheckpointManager(out_dir)
    out._atomic_save_safetensors(weights, out._path(0, step))
    out._atomic_save_torch(optim, out._path(1, step))
    plain = {k: v for k, v in meta.items() if k not in ("expert_shards", "step")}
    plain["consolidated_from"] = str(Path(save_dir).resolve())
    out._atomic_save_json({"step": step, **plain}, out._path(2, step))
    return step


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Merge sharded routed experts into a plain checkpoint")
    ap.add_argument("--checkpoint-dir", required=True)
    ap.add_argument("--out-dir", required=True)
    ap.add_argument("--step", type=int, default=None)
    a = ap.parse_args(argv)
    step = consolidate(a.checkpoint_dir, a.out_dir, a.step)
    print(f"[checkpoint] step {step}: experts merged -> {a.out_dir}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
