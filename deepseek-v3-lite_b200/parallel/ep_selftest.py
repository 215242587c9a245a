"""Correctness check of the expert-parallel MoE path on the GPUs of one box.

``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
-m parallel.ep_selftest`` (from ``deepseek-v3-lite_b200/``; N = 1..8) runs a
routed-expert layer forward + backward through the peer-memory dispatch /
combine kernels on every rank, twice (so the signal counters advance across
calls), and compares each rank's outputs, token gradients, gate-weight
gradients and expert weight gradients with an fp32 PyTorch evaluation of the
same layer over the tokens of all ranks, in both receive layouts (balanced:
the ranks' partial expert gradients summed; owner: each rank's own experts).  Exits non-zero on mismatch.
Run without torchrun it checks the single-rank path (the rank stores into its
own heap through the same kernels).  ``--engine`` instead trains the same tiny
model with experts spread over the ranks and with experts replicated and
compares losses and averaged gradients.  ``--shard`` compares expert-parallel
training with the routed experts' weights, gradients and optimizer state
sharded over the ranks against the same training with them replicated: three
optimizer steps on identical synthetic gradients (with the peer-memory and
with the NCCL data-parallel step), one real step, and a checkpoint round
trip through the trainer.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.nn.functional as F


def make_case(E, k, D, I, T, rank, device):
    """Identical expert weights on every rank; rank-specific tokens and grads."""
    g = torch.Generator(device="cpu").manual_seed(1234)
    w1 = (torch.randn(E, I, D, generator=g) * 0.05)
    w3 = (torch.randn(E, I, D, generator=g) * 0.05)
    w2 = (torch.randn(E, D, I, generator=g) * 0.05)
    gate = torch.randn(E, D, generator=g) * 0.05
    gr = torch.Generator(device="cpu").manual_seed(100 + rank)
    x = torch.randn(T, D, generator=gr)
    dout = torch.randn(T, D, generator=gr) * 0.1
    to = dict(device=device)
    return (w1.to(**to), w3.to(**to), w2.to(**to), gate.to(**to), x.to(**to).bfloat16(),
            dout.to(**to).bfloat16())


def reference_layer(x, idx, wts, dout, w1, w3, w2):
    """fp32 y[t] = sum_j w[t,j] * W2_e (silu(W1_e x) * W3_e x) and its gradients."""
    xs = x.float().detach().requires_grad_(True)
    ws = wts.float().detach().requires_grad_(True)
    p1, p3, p2 = (w.detach().clone().requires_grad_(True) for w in (w1, w3, w2))
    y = torch.zeros_like(xs)
    for e in range(p1.shape[0]):
        rows, slots = (idx.long() == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        xe = xs[rows]
        h = F.silu(xe @ p1[e].t()) * (xe @ p3[e].t())
        y = y.index_add(0, rows, ws[rows, slots].unsqueeze(1) * (h @ p2[e].t()))
    y.backward(dout.float())
    return y.detach(), xs.grad, ws.grad, p1.grad, p3.grad, p2.grad


def run(E=8, k=2, D=256, I=128, T=512, iters=2, verbose=True, balanced=True) -> bool:
    """Layer check in one receive layout (``balanced`` or owner).  In the
    balanced layout each rank holds partial weight gradients of every expert
    its share touches; their sum over ranks is compared with the reference."""
    sys.path.insert(0, __file__.rsplit("/parallel/", 1)[0])
    import torch.distributed as dist
    from ops._ext import native
    from parallel.dist import init_distributed
    from parallel.ep import ExpertParallel, moe_backward_ep, moe_forward_ep

    rank, world, device = init_distributed(timeout_s=60)
    C = native()
    C.status_reset()
    w1, w3, w2, gate, x, dout = make_case(E, k, D, I, T, rank, device)
    w13 = torch.stack([w1, w3], 1).bfloat16().contiguous()            # [E, 2, I, D]
    w2b = w2.bfloat16().contiguous()
    logits = torch.zeros(T, (E + 7) // 8 * 8, device=device)
    C.linear_fwd(x, gate.bfloat16(), logits[:, :E], False)
    idx = torch.empty(T, k, dtype=torch.int32, device=device)
    wts = torch.empty(T, k, device=device)
    ssel = torch.empty(T, k, device=device)
    counts = torch.zeros(E, dtype=torch.int32, device=device)
    C.router_topk(logits, torch.zeros(E, device=device), E, k, 1.0, idx, wts, ssel, counts)

    ep = ExpertParallel(E, k, D, T, n_slots=2, timeout_s=20, balanced=balanced)
    lo, hi = ep.g_lo, ep.g_lo + ep.G          # weight groups of the layout
    ok = True
    # every rank's tokens for the owned-expert weight-gradient reference
    if world > 1:
        gath = []
        for t in (x, idx, wts, dout):
            buf = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(buf, t.contiguous())
            gath.append(torch.cat(buf, 0))
        x_all, idx_all, w_all, d_all = gath
    else:
        x_all, idx_all, w_all, d_all = x, idx, wts, dout
    w1r, w3r, w2r = (w.bfloat16().float() for w in (w1, w3, w2))
    y_ref, dx_ref, dw_ref, _, _, _ = reference_layer(x, idx, wts, dout, w1r, w3r, w2r)
    _, _, _, g1_ref, g3_ref, g2_ref = reference_layer(x_all, idx_all, w_all, d_all, w1r, w3r, w2r)

    def close(name, a, b, tol):
        nonlocal ok
        err = (a.float() - b.float()).norm() / max(b.float().norm().item(), 1e-12)
        if not (err <= tol):
            ok = False
            print(f"[rank {rank}] {name}: relative error {err:.3e} > {tol}", flush=True)
        elif verbose:
            print(f"[rank {rank}] {name}: relative error {err:.3e}", flush=True)

    for it in range(iters):
        slot = it % 2
        out = torch.zeros(T, D, device=device)
        ctx = moe_forward_ep(ep, slot, x, idx, wts, counts, w13[lo:hi], w2b[lo:hi], out, I)
        dx = torch.zeros(T, D, device=device)
        g13 = torch.zeros(hi - lo, 2 * I, D, device=device)
        g2 = torch.zeros(hi - lo, D, I, device=device)
        dw = moe_backward_ep(ep, ctx, dout, w13[lo:hi], w2b[lo:hi], g13, g2, dx, I).clone()
        torch.cuda.synchronize()
        if balanced and world > 1:
            for gbuf in (g13, g2):               # partial per rank; the sum is the gradient
                dist.all_reduce(gbuf)
        cnt_global = ctx["cnt_all"].sum(0)
        expect_global = torch.bincount(idx_all.long().flatten(), minlength=E).to(cnt_global)
        if not torch.equal(cnt_global, expect_global):
            ok = False
            print(f"[rank {rank}] exchanged counts differ from the all-gathered routing", flush=True)
        tag = f"{'balanced' if balanced else 'owner'} it{it}"
        close(f"{tag} y", out, y_ref, 2e-2)
        close(f"{tag} dx", dx, dx_ref, 3e-2)
        close(f"{tag} dw", dw, dw_ref, 3e-2)
        close(f"{tag} dW1", g13[:, :I], g1_ref[lo:hi], 3e-2)
        close(f"{tag} dW3", g13[:, I:], g3_ref[lo:hi], 3e-2)
        close(f"{tag} dW2", g2, g2_ref[lo:hi], 3e-2)
    code = C.status_read()
    if code:
        ok = False
        print(f"[rank {rank}] device status word {code}", flush=True)
    ep.close()
    return ok


ENGINE_CFG = {
    "vocab_size": 1000, "dim": 256, "n_layers": 3, "n_heads": 4, "n_dense_layers": 1,
    "n_routed_experts": 8, "n_shared_experts": 1, "n_activated_experts": 2, "inter_dim": 512,
    "moe_inter_dim": 128, "kv_lora_rank": 64, "q_lora_rank": 0, "qk_nope_head_dim": 48,
    "qk_rope_head_dim": 16, "v_head_dim": 64, "max_seq_len": 128, "rope_theta": 10000,
    "rope_factor": 1.0, "mscale": 1.0, "mtp_depth": 1, "mtp_loss_weight": 0.3,
    "attn_impl": "sdpa", "weight_tying": True,
}


def run_engine(verbose=True) -> bool:
    """The training engine with experts spread over the ranks vs the same
    engine with experts replicated: same losses, same averaged gradients."""
    import copy
    import torch.distributed as dist
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    from ops.engine import TrainEngine
    from parallel.dist import init_distributed
    from training.pretrain import TrainingConfig, _unique_params

    rank, world, device = init_distributed(timeout_s=60)
    torch.manual_seed(0)
    base = Transformer(dict(ENGINE_CFG)).to(device)
    for moe in base.moe_layers():
        moe.gate.weight.data.mul_(40.0)   # spread the router scores (no near-ties)
    base_mtp = MultiTokenPrediction(dict(ENGINE_CFG), base).to(device)
    engines = []
    for ep_size in (1, 0):
        mtp = copy.deepcopy(base_mtp)
        model = mtp.main_model
        params = _unique_params(mtp)
        groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
                  {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
        engines.append(TrainEngine(model, mtp, TrainingConfig(lr=1e-3, ep_size=ep_size, batch_size=4), groups))
    B, S = 4, 128
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    tokens = torch.randint(0, ENGINE_CFG["vocab_size"], (B, S), generator=g).to(device)
    targets = torch.randint(0, ENGINE_CFG["vocab_size"], (B, S), generator=g).to(device)
    ok = True
    outs = []
    for eng in engines:
        eng.zero_grad()
        for _ in range(2):   # second pass replays the captured graph
            eng.zero_grad()
            out = eng.forward_backward(tokens, targets, loss_scale=1.0)
        torch.cuda.synchronize()
        eng.check()
        eng.dp.reduce_gradients()
        outs.append((out["loss"].item(), [f.grad.clone() for f in eng.flats]))
    (l0, g0), (l1, g1) = outs
    if abs(l0 - l1) > 1e-3 * max(1.0, abs(l0)):
        ok = False
        print(f"[rank {rank}] loss {l0} (replicated experts) vs {l1} (expert parallel)", flush=True)
    for i, (a, b) in enumerate(zip(g0, g1)):
        err = ((a - b).norm() / a.norm().clamp_min(1e-12)).item()
        if verbose:
            print(f"[rank {rank}] flat grad {i}: relative difference {err:.3e}", flush=True)
        if not err < 2e-2:
            ok = False
    for eng in engines:
        eng.close()
    return ok


def run_shard(verbose=True) -> bool:
    """Expert-parallel training with routed experts sharded over the ranks
    (``ep_shard_experts``) vs replicated: identical weights, norms, losses."""
    import copy
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    from ops.engine import TrainEngine
    from parallel.dist import init_distributed
    from parallel.ep import expert_range
    from training.pretrain import TrainingConfig, _unique_params

    rank, world, device = init_distributed(timeout_s=60)
    torch.manual_seed(0)
    base = Transformer(dict(ENGINE_CFG)).to(device)
    for moe in base.moe_layers():
        moe.gate.weight.data.mul_(40.0)
    base_mtp = MultiTokenPrediction(dict(ENGINE_CFG), base).to(device)
    ok = True

    def engine(shard):
        mtp = copy.deepcopy(base_mtp)
        params = _unique_params(mtp)
        names = {id(p): n for n, p in mtp.named_parameters()}
        groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
                  {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
        eng = TrainEngine(mtp.main_model, mtp, TrainingConfig(lr=1e-3, ep_size=0, batch_size=4,
                                                               ep_shard_experts=shard), groups)
        assert eng.shard_experts == (shard and world > 1)
        return eng, [(names[id(p)], p) for p in params]

    def owned(eng, name):
        """(is a routed expert, owned by this rank)"""
        if ".experts." not in name:
            return False, True
        e = int(name.split(".experts.")[1].split(".")[0])
        lo, hi = expert_range(rank, ENGINE_CFG["n_routed_experts"], world)
        return True, lo <= e < hi

    def masters(eng, params):
        out = {}
        for name, p in params:
            is_exp, mine = owned(eng, name)
            if mine:
                out[name] = eng._fl(p).view(eng._fl(p).master, p).clone()
        return out

    # (a) synthetic gradients: replicated parameters get rank-specific values,
    # a routed expert's gradient is its owner's (zero on the other ranks)
    res = {}
    modes = {"sharded": (True, "0"), "sharded, NCCL step": (True, "1"), "replicated": (False, "0")}
    for mode, (shard, nccl) in modes.items():
        saved_env = os.environ.get("DSV3_DP_NCCL")
        os.environ["DSV3_DP_NCCL"] = nccl
        try:
            eng, params = engine(shard)
        finally:
            if saved_env is None:
                os.environ.pop("DSV3_DP_NCCL", None)
            else:
                os.environ["DSV3_DP_NCCL"] = saved_env
        for step in range(3):
            for f in eng.flats:
                f.grad.zero_()
            for i, (name, p) in enumerate(params):
                is_exp, mine = owned(eng, name)
                if not mine:
                    continue
                gen = torch.Generator(device="cpu").manual_seed(100000 * step + 10 * i + (0 if is_exp else 1 + rank))
                fl = eng._fl(p)
                fl.view(fl.grad, p).copy_(torch.randn(p.shape, generator=gen) * 1e-2)
            eng.clip_and_step(1.0 if step != 1 else 1e-3)
        torch.cuda.synchronize()
        eng.check()
        res[mode] = (masters(eng, params), float(eng.optimizer.grad_norm))
        eng.close()
    m0, n0 = res["replicated"]
    for mode in ("sharded", "sharded, NCCL step"):
        m1, n1 = res[mode]
        worst = max((m0[k] - m1[k]).abs().max().item() for k in m1)
        if verbose:
            print(f"[rank {rank}] synthetic steps: max |replicated - {mode}| {worst:.3e}, norms {n0:.6f} / {n1:.6f}",
                  flush=True)
        if not (worst <= 1e-5 and abs(n0 - n1) <= 1e-5 * max(1.0, n0)):
            ok = False

    # (b) one real step from the same weights: same loss, norm and update
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    tok = torch.randint(0, ENGINE_CFG["vocab_size"], (4, 129), generator=g).to(device)
    res = {}
    for shard in (False, True):
        eng, params = engine(shard)
        out = eng.forward_backward(tok[:, :-1], tok[:, 1:], loss_scale=1.0)
        eng.clip_and_step(1.0)
        torch.cuda.synchronize()
        eng.check()
        res[shard] = (out["loss"].item(), float(eng.optimizer.grad_norm), masters(eng, params))
        eng.close()
    (l0, n0, m0), (l1, n1, m1) = res[False], res[True]
    worst = max((m0[k] - m1[k]).abs().max().item() for k in m1)
    if verbose:
        print(f"[rank {rank}] real step: loss {l0:.6f} / {l1:.6f}, norm {n0:.6f} / {n1:.6f}, "
              f"max weight difference {worst:.3e}", flush=True)
    if not (abs(l0 - l1) <= 1e-5 * max(1.0, abs(l0)) and abs(n0 - n1) <= 1e-4 * max(1.0, n0) and worst <= 1e-5):
        ok = False

    # (c) checkpoint round trip through the trainer: per-rank expert shards,
    # then a fresh trainer resumes and repeats the next step exactly
    import shutil
    import tempfile
    import torch.distributed as dist
    from training.pretrain import Pretrainer
    box = [tempfile.mkdtemp(prefix="dsv3_shard_ckpt_") if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    ckdir = box[0]

    def trainer():
        cfg = TrainingConfig(model_config=dict(ENGINE_CFG), checkpoint_dir=ckdir, vocab_size=ENGINE_CFG["vocab_size"],
                             max_seq_len=128, batch_size=4, gradient_accumulation_steps=1, warmup_steps=2,
                             lr=1e-3, mtp_weight=0.3, grad_checkpoint=False, compile_model=False,
                             log_per_component_params=False, ep_size=0, ep_shard_experts=True)
        return Pretrainer(cfg)

    toks = [torch.randint(0, ENGINE_CFG["vocab_size"], (4, 129), generator=g).to(device) for _ in range(3)]
    tr = trainer()
    for i in range(2):
        tr.train_step(toks[i][:, :-1], toks[i][:, 1:], i)
    tr.save_checkpoint(2)
    want = float(tr.train_step(toks[2][:, :-1], toks[2][:, 1:], 2)["loss"])
    tr.engine.close()
    tr2 = trainer()
    tr2.load_checkpoint(2)
    got = float(tr2.train_step(toks[2][:, :-1], toks[2][:, 1:], 2)["loss"])
    tr2.engine.close()
    shards = sorted(p.name for p in __import__("pathlib").Path(ckdir).glob("experts_step_2_*"))
    if verbose:
        print(f"[rank {rank}] resume: loss {want:.6f} before / {got:.6f} after; shard files {shards}", flush=True)
    if not (abs(want - got) <= 1e-5 * max(1.0, abs(want)) and len(shards) == world):
        ok = False
    dist.barrier()
    if rank == 0:
        shutil.rmtree(ckdir, ignore_errors=True)
    return ok


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--engine", action="store_true", help="compare the training engine with and without EP")
    ap.add_argument("--shard", action="store_true", help="compare sharded with replicated routed experts")
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--inter", type=int, default=128)
    ap.add_argument("--tokens", type=int, default=512)
    a = ap.parse_args()
    if a.shard:
        ok = run_shard()
    elif a.engine:
        ok = run_engine()
    else:
        ok = all([run(a.experts, a.topk, a.dim, a.inter, a.tokens, balanced=b) for b in (True, False)])
    import torch.distributed as dist
    if dist.is_initialized():
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
        dist.destroy_process_group()
    print("EP_SELFTEST", "OK" if ok else "FAILED", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
