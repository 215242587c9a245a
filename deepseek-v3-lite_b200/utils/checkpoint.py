"""Step-numbered, crash-safe checkpoints in the reference's on-disk format.

One checkpoint is three files in ``save_dir`` (reference
``utils/checkpoint.py:11-110``):

* ``model_step_N.safetensors`` - the state dict, one key per *storage*
  (tied tensors are written once: the first key in iteration order wins);
* ``optim_step_N.pt`` - ``torch.save`` of the optimizer state dict;
* ``meta_step_N.json`` - ``{"step": N, ...}``; the file name's step wins over
  a caller-supplied ``step``.

Each file is written to a temporary file in the same directory and moved into
place with ``os.replace``, so a crash leaves either the old file or none.  A
step counts as present only when all three files exist.

Training with routed experts sharded over the ranks adds one file per rank,
``experts_step_N_rankRofW.safetensors``: that rank's routed-expert weights
under their state-dict names plus their AdamW moments under ``exp_avg.`` /
``exp_avg_sq.`` prefixes; the model file then holds everything else and the
metadata records ``"expert_shards": W``.  Such a step counts as present only
when all W shard files exist too.  Loading into an unsharded model merges the
shards' weights (``merge_expert_shards``).
"""
from __future__ import annotations

import contextlib
import json
import logging
import os
import tempfile
import threading
from pathlib import Path
from typing import Dict, Optional

import torch
from safetensors.torch import load_file, save_file

log = logging.getLogger(__name__)

_FILES = ("model_step_{}.safetensors", "optim_step_{}.pt", "meta_step_{}.json")
_SHARD = "experts_step_{}_rank{}of{}.safetensors"
_MOMENT_PREFIXES = ("exp_avg.", "exp_avg_sq.")


def _to_host(obj):
    """Copy every tensor inside nested dicts / lists / tuples to host memory."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _to_host(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_host(v) for v in obj)
    return obj


class CheckpointManager:
    """Save and restore model / optimizer / metadata triples by step."""

    def __init__(self, save_dir: str):
        self.save_dir = Path(save_dir)
        self.save_dir.mkdir(parents=True, exist_ok=True)
        self._writer: Optional[threading.Thread] = None
        self._writer_error: Optional[BaseException] = None

    # ------------------------------------------------------------------ paths
    def _path(self, kind: int, step: int) -> Path:
        return self.save_dir / _FILES[kind].format(step)

    def _list_steps(self) -> list:
        steps = []
        for p in self.save_dir.glob("model_step_*.safetensors"):
            tail = p.stem.rsplit("_", 1)[-1]
            if tail.isdigit():
                steps.append(int(tail))
        return steps

    def expert_shard_path(self, step: int, rank: int, world: int) -> Path:
        return self.save_dir / _SHARD.format(step, rank, world)

    def _meta(self, step: int) -> dict:
        try:
            with open(self._path(2, step)) as f:
                return json.load(f)
        except (OSError, ValueError):
            return {}

    def _checkpoint_complete(self, step: int) -> bool:
        if not all(self._path(i, step).exists() for i in range(3)):
            return False
        w = int(self._meta(step).get("expert_shards", 0) or 0)
        return all(self.expert_shard_path(step, r, w).exists() for r in range(w))

    def latest_step(self) -> Optional[int]:
        """Newest step whose three files all exist, or ``None``."""
        complete = [s for s in self._list_steps() if self._checkpoint_complete(s)]
        return max(complete) if complete else None

    # ------------------------------------------------------------------- save
    @contextlib.contextmanager
    def _atomic_write(self, path: Path, suffix: str):
        fd, tmp = tempfile.mkstemp(dir=self.save_dir, suffix=suffix)
        os.close(fd)
        try:
            yield tmp
            os.replace(tmp, path)
        except BaseException:
            with contextlib.suppress(OSError):
                os.unlink(tmp)
            raise

    @staticmethod
    def _unique_storage(state: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        seen, out = set(), {}
        for key, t in state.items():
            ptr = t.data_ptr()
            if ptr in seen:
                continue
            seen.add(ptr)
            out[key] = t.detach().contiguous()
        return out

    def _atomic_save_safetensors(self, state: dict, path: Path) -> None:
        tensors = self._unique_storage(state)
        with self._atomic_write(path, ".safetensors.tmp") as tmp:
            save_file(tensors, tmp)

    def _atomic_save_torch(self, obj, path: Path) -> None:
        with self._atomic_write(path, ".pt.tmp") as tmp:
            torch.save(obj, tmp)

    def _atomic_save_json(self, obj: dict, path: Path) -> None:
        with self._atomic_write(path, ".json.tmp") as tmp:
            with open(tmp, "w") as f:
                json.dump(obj, f, indent=2, default=str)

    def save(self, model: torch.nn.Module, optimizer, step: int, extra_meta: Optional[dict] = None,
             state_dict: Optional[dict] = None, optimizer_state: Optional[dict] = None,
             background: bool = False) -> None:
        """Write the three files for ``step``.

        ``state_dict`` overrides ``model.state_dict()``; ``optimizer_state``
        overrides ``optimizer.state_dict()`` (used by sharded optimizers that
        gather to the reference layout first).  With ``background`` the
        tensors are first copied to host memory (a consistent snapshot of this
        step) and a writer thread writes the files while the caller goes on;
        one save is in flight at a time (a new one, a load or ``wait()`` waits
        for it).  The metadata file is written last either way, so a step is
        never reported complete before all of its files exist.
        """
        state = state_dict if state_dict is not None else model.state_dict()
        opt_state = optimizer_state if optimizer_state is not None else optimizer.state_dict()
        meta = {k: v for k, v in (extra_meta or {}).items() if k != "step"}
        if not background:
            self._write(step, state, opt_state, meta)
            return
        self.wait()
        snap_state = {k: v.detach().to("cpu", copy=True) for k, v in self._unique_storage(state).items()}
        snap_opt = _to_host(opt_state)
        self._writer_error = None
        self._writer = threading.Thread(target=self._write_guarded, args=(step, snap_state, snap_opt, meta),
                                        name=f"checkpoint-{step}")
        self._writer.start()

    def _write(self, step: int, state: dict, opt_state, meta: dict) -> None:
        self._atomic_save_safetensors(state, self._path(0, step))
        self._atomic_save_torch(opt_state, self._path(1, step))
        self._atomic_save_json({"step": step, **meta}, self._path(2, step))
        log.info("[checkpoint] saved step %d -> %s", step, self.save_dir)

    def _write_guarded(self, step: int, state: dict, opt_state, meta: dict) -> None:
        try:
            self._write(step, state, opt_state, meta)
        except BaseException as exc:  # reported by wait()
            self._writer_error = exc

    def wait(self) -> None:
        """Block until a background save finished; re-raise its error."""
        if self._writer is not None:
            self._writer.join()
            self._writer = None
        if self._writer_error is not None:
            err, self._writer_error = self._writer_error, None
            raise RuntimeError("background checkpoint write failed") from err

    def save_expert_shard(self, step: int, rank: int, world: int, tensors: Dict[str, torch.Tensor]) -> None:
        """Write one rank's routed experts (weights and prefixed moments).
        Every entry is copied to host memory first (the device tensors are
        views into flat buffers)."""
        host = {k: v.detach().to("cpu", copy=True).contiguous() for k, v in tensors.items()}
        with self._atomic_write(self.expert_shard_path(step, rank, world), ".safetensors.tmp") as tmp:
            save_file(host, tmp)

    def load_expert_shard(self, step: int, rank: int, world: int, device: str = "cpu") -> Dict[str, torch.Tensor]:
        path = self.expert_shard_path(step, rank, world)
        if not path.exists():
            raise FileNotFoundError(f"expert shard not found: {path}")
        return load_file(str(path), device=str(device))

    def expert_shard_weights(self, step: int, device: str = "cpu") -> Dict[str, torch.Tensor]:
        """The routed-expert weights of every shard of ``step`` (no moments)."""
        w = int(self._meta(step).get("expert_shards", 0) or 0)
        out: Dict[str, torch.Tensor] = {}
        for r in range(w):
            for k, v in self.load_expert_shard(step, r, w, device).items():
                if not k.startswith(_MOMENT_PREFIXES):
                    out[k] = v
        return out

    # ------------------------------------------------------------------- load
    def load(self, model: torch.nn.Module, step: int, device: str = "cuda", optimizer=None,
             strict: bool = True, merge_expert_shards: bool = True) -> dict:
        """Restore ``step`` into ``model`` (and ``optimizer``); return the metadata.

        With ``strict`` a missing or unexpected key raises ``RuntimeError``;
        otherwise it is logged.  A step saved with sharded experts has its
        shards' weights merged in unless ``merge_expert_shards`` is false (a
        sharded run loads its own shard instead).
        """
        self.wait()
        wpath = self._path(0, step)
        if not wpath.exists():
            raise FileNotFoundError(f"Checkpoint not found: {wpath}\nAvailable steps: {sorted(self._list_steps())}")
        weights = load_file(str(wpath), device=str(device))
        if merge_expert_shards:
            weights.update(self.expert_shard_weights(step, device=str(device)))
        missing, unexpected = model.load_state_dict(weights, strict=False)
        for what, keys in (("missing", missing), ("unexpected", unexpected)):
            if not keys:
                continue
            msg = f"[checkpoint] {len(keys)} {what} key(s): {list(keys)[:5]}{'...' if len(keys) > 5 else ''}"
            if strict:
                raise RuntimeError(msg)
            log.warning(msg)
        if optimizer is not None:
            opath = self._path(1, step)
            if opath.exists():
                optimizer.load_state_dict(torch.load(opath, map_location=device, weights_only=True))
            else:
                log.warning("[checkpoint] no optimizer state at %s; optimizer starts fresh", opath)
        mpath = self._path(2, step)
        if mpath.exists():
            with open(mpath) as f:
                return json.load(f)
        return {"step": step}
