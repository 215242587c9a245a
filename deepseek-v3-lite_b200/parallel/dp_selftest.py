"""Correctness check of the peer-memory data-parallel optimizer step.

``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
-m parallel.dp_selftest`` (from ``deepseek-v3-lite_b200/``) trains the same
tiny model's optimizer through three steps with the same rank-specific
synthetic gradients, once with the NCCL all-reduce step and once with the
fused reduce-scatter / sharded AdamW / all-gather step over peer memory, and
checks that both give the same weights, gradient norm (one step clips) and
second moments; checks that the fused step keeps only this rank's shard of
the AdamW moments (ZeRO-1) and that the learning rate it applies at optimizer
steps 1..N is the single-process ``LambdaLR`` schedule, with no scheduler
ordering warning; then trains two real steps with the fused step and checks
that every rank holds bit-identical weights.  Exits non-zero on mismatch.
"""
from __future__ import annotations

import copy
import os
import sys

import torch

from parallel.ep_selftest import ENGINE_CFG


def run(verbose: bool = True) -> bool:
    import torch.distributed as dist
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    from ops.engine import TrainEngine
    from parallel.dist import init_distributed
    from training.pretrain import TrainingConfig, _unique_params

    rank, world, device = init_distributed(timeout_s=60)
    torch.manual_seed(0)
    base = Transformer(dict(ENGINE_CFG)).to(device)
    base_mtp = MultiTokenPrediction(dict(ENGINE_CFG), base).to(device)
    ok = True

    def engine(mode):
        os.environ["DSV3_DP_NCCL"] = "1" if mode == "nccl" else "0"
        mtp = copy.deepcopy(base_mtp)
        params = _unique_params(mtp)
        groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
                  {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
        eng = TrainEngine(mtp.main_model, mtp, TrainingConfig(lr=1e-3, batch_size=4), groups)
        assert (mode == "fused") == hasattr(eng.dp, "step"), "unexpected data-parallel implementation"
        return eng

    # (a) identical rank-specific gradients through both optimizer steps
    results = {}
    for mode in ("nccl", "fused"):
        eng = engine(mode)
        for step in range(3):
            gen = torch.Generator(device="cpu").manual_seed(1000 * step + rank)
            for f in eng.flats:
                f.grad.copy_(torch.randn(f.numel, generator=gen) * 1e-2)
            eng.clip_and_step(1.0 if step != 1 else 1e-3)   # step 1 clips
        torch.cuda.synchronize()
        eng.check()
        sd = eng.optimizer_state_for_checkpoint()
        moments = torch.cat([st["exp_avg_sq"].flatten() for st in sd["state"].values()])
        results[mode] = ([f.master.clone() for f in eng.flats], float(eng.optimizer.grad_norm), moments)
        eng.close()
    (m0, n0, v0), (m1, n1, v1) = results["nccl"], results["fused"]
    for i, (a, b) in enumerate(zip(m0, m1)):
        diff = (a - b).abs().max().item()
        if verbose:
            print(f"[rank {rank}] flat {i}: max |nccl - fused| after 3 steps = {diff:.3e}", flush=True)
        if not diff <= 1e-5:
            ok = False
    if abs(n0 - n1) > 1e-5 * max(1.0, n0):
        ok = False
        print(f"[rank {rank}] grad norms differ: {n0} vs {n1}", flush=True)
    mdiff = ((v0 - v1).norm() / v0.norm().clamp_min(1e-30)).item()
    if verbose:
        print(f"[rank {rank}] second moments relative difference {mdiff:.3e}", flush=True)
    if not mdiff < 1e-5:
        ok = False

    # (b) ZeRO-1 moments and the learning-rate schedule under the fused step
    import warnings
    from torch.optim.lr_scheduler import LambdaLR
    from training.pretrain import make_warmup_cosine_lambda
    eng = engine("fused")
    opt = eng.optimizer
    replicated = sum(f.numel for f in eng.flats[:eng.dp.n_heap])
    held = sum(m.numel() for m in opt.exp_avg[:eng.dp.n_heap])
    expect = sum(hi - lo for lo, hi in eng.dp.shards)
    if verbose:
        print(f"[rank {rank}] AdamW moments held for replicated parameters: {8 * held:,} bytes "
              f"(unsharded: {8 * replicated:,})", flush=True)
    if held != expect or (world > 1 and held >= replicated):
        ok = False
        print(f"[rank {rank}] moment shard holds {held} elements, expected {expect}", flush=True)
    lam = make_warmup_cosine_lambda(3, 10, 0.1)
    sched = LambdaLR(opt, lam)
    applied = []
    inner = opt.stepper

    def recording(o):
        applied.append([float(g["lr"]) for g in o.param_groups])
        inner(o)
    opt.stepper = recording
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        for _ in range(6):
            for f in eng.flats:
                f.grad.normal_(0, 1e-2)
            eng.clip_and_step(1.0)
            sched.step()
    expected = [[1e-3 * lam(k)] * len(opt.param_groups) for k in range(6)]
    if any(abs(a - b) > 1e-12 for ra, rb in zip(applied, expected) for a, b in zip(ra, rb)) or len(applied) != 6:
        ok = False
        print(f"[rank {rank}] learning rates applied {applied} != schedule {expected}", flush=True)
    if any("lr_scheduler.step()" in str(w.message) for w in caught):
        ok = False
        print(f"[rank {rank}] scheduler ordering warning raised", flush=True)
    torch.cuda.synchronize()
    eng.check()
    eng.close()

    # (c) real training steps: finite losses, identical weights on every rank
    eng = engine("fused")
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    for _ in range(2):
        for _ in range(2):
            tok = torch.randint(0, ENGINE_CFG["vocab_size"], (4, 129), generator=g).to(device)
            out = eng.forward_backward(tok[:, :-1], tok[:, 1:], loss_scale=0.5)
        eng.clip_and_step(1.0)
        eng.zero_grad()
    torch.cuda.synchronize()
    eng.check()
    if not torch.isfinite(out["loss"]).item():
        ok = False
    if world > 1:
        for f in eng.flats:
            for buf in (f.master, f.shadow):
                ref = buf.clone()
                dist.broadcast(ref, src=0)
                if not torch.equal(ref, buf):
                    ok = False
                    print(f"[rank {rank}] weights differ from rank 0 after the fused step", flush=True)
    eng.close()
    return ok


def main() -> None:
    ok = run()
    import torch.distributed as dist
    if dist.is_initialized():
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
        dist.destroy_process_group()
    print("DP_SELFTEST", "OK" if ok else "FAILED", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
