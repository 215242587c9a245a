"""MoE-layer microbenchmark under expert parallelism.

``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
-m parallel.bench_ep [--tokens 16384] [--sweep] [--impl ours|reference]``
(from ``deepseek-v3-lite_b200/``) times forward + backward of one DeepSeekMoE
layer with hidden 2048, 64 routed SwiGLU experts of width 1408 (top-6) and 2
shared experts, bf16, hidden states N(0, 1), router weights N(0, 0.02), bias
0, the routed experts spread over the N ranks (EP = N), ``--tokens`` tokens
per rank.

ours       router GEMM + top-k kernel, peer-memory count exchange and
           dispatch, grouped tcgen05 SwiGLU / down GEMMs, peer-memory combine,
           and the mirrored backward with all weight gradients.
reference  the reference's own modules (``AuxLossFreeGate``, ``Expert``;
           models/moe.py:7-49 of the reference tree) under bf16 autocast,
           wrapped in an NCCL ``all_to_all_single`` dispatch / combine harness
           (the reference has no multi-GPU code of its own).

Time: CUDA events on every rank after warm-up, max over ranks.  Per rank the
line also reports the bytes that crossed NVLink (rows sent to other ranks in
the four transfer phases) and, for ours, the device time of each transfer
phase (the shared experts run on a side stream meanwhile, so a phase also
holds the wait for the slowest peer) and its fraction of the NVLink roofline
(bytes / 770 GB/s per direction,
the peer-copy bandwidth measured on this kind of box), and the whole layer's
fraction of its roofline: the slower of its FLOPs at the measured bf16 peak
and its bytes at that link bandwidth.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
NVLINK_GBS = 770.0          # measured peer copy, GB/s per direction per GPU
D, E, TOPK, INTER, N_SHARED = 2048, 64, 6, 1408, 2


def _peaks():
    for p in (HERE.parent.parent / "MEASURED_PEAKS.json",):
        if p.exists():
            d = json.loads(p.read_text())
            return float(d.get("bf16_tflops", 1590.0)), float(d.get("hbm_gbs", 6650.0)), "measured"
    return 1590.0, 6650.0, "fallback"


def _flops(T: int) -> float:
    routed = T * TOPK * 2.0 * D * INTER * 3      # gate, up, down per routed row
    shared = T * N_SHARED * 2.0 * D * INTER * 3
    router = T * 2.0 * D * E
    return 3.0 * (routed + shared + router)      # forward + (data + weight) gradients


def _max_over_ranks(v: float) -> float:
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time(fn, warmup: int, iters: int):
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


# --------------------------------------------------------------------- ours
class OursLayer:
    def __init__(self, T: int, rank: int, world: int, device):
        from ops._ext import native
        from parallel.ep import ExpertParallel
        self.C = native()
        self.T = T
        g = torch.Generator(device="cpu").manual_seed(0)
        bf = dict(device=device, dtype=torch.bfloat16)
        self.gate = (torch.randn(E, D, generator=g) * 0.02).to(**bf)
        self.bias = torch.zeros(E, device=device)
        self.ep = ExpertParallel(E, TOPK, D, T, n_slots=1,
                                 balanced=os.environ.get("DSV3_EP_BALANCED", "1") != "0")
        # weight groups of the layout: all experts (balanced) or the owned ones
        lo, hi = self.ep.g_lo, self.ep.g_lo + self.ep.G
        std = 1.0 / D ** 0.5
        self.w13 = (torch.randn(hi - lo, 2, INTER, D, generator=g) * std).to(**bf)
        self.w2 = (torch.randn(hi - lo, D, INTER, generator=g) * (1.0 / INTER ** 0.5)).to(**bf)
        self.sw13 = [(torch.randn(1, 2, INTER, D, generator=g) * std).to(**bf) for _ in range(N_SHARED)]
        self.sw2 = [(torch.randn(D, INTER, generator=g) * (1.0 / INTER ** 0.5)).to(**bf) for _ in range(N_SHARED)]
        f32 = dict(device=device, dtype=torch.float32)
        self.g13 = torch.zeros(hi - lo, 2 * INTER, D, **f32)
        self.g2 = torch.zeros(hi - lo, D, INTER, **f32)
        self.sg13 = [torch.zeros(2 * INTER, D, **f32) for _ in range(N_SHARED)]
        self.sg2 = [torch.zeros(D, INTER, **f32) for _ in range(N_SHARED)]
        self.ggate = torch.zeros(E, D, **f32)
        gx = torch.Generator(device="cpu").manual_seed(100 + rank)
        self.x = torch.randn(T, D, generator=gx).to(**bf)
        self.dout = (torch.randn(T, D, generator=gx) * 0.01).to(**bf)
        self.empty_i32 = torch.empty(0, dtype=torch.int32, device=device)
        self.events = None

    def _mark(self, name):
        if self.events is not None:
            ev = torch.cuda.Event(True)
            ev.record()
            self.events.append((name, ev))

    def step(self):
        from parallel.ep import moe_backward_ep, moe_forward_ep
        C, T, dev = self.C, self.T, self.x.device
        x = self.x
        self._mark("start")
        logits = torch.empty(T, E, device=dev)
        C.linear_fwd(x, self.gate, logits, False)
        idx = torch.empty(T, TOPK, dtype=torch.int32, device=dev)
        wts = torch.empty(T, TOPK, device=dev)
        ssel = torch.empty(T, TOPK, device=dev)
        counts = torch.zeros(E, dtype=torch.int32, device=dev)
        C.router_topk(logits, self.bias, E, TOPK, 1.0, idx, wts, ssel, counts)
        out = torch.zeros(T, D, device=dev)
        dx = torch.zeros(T, D, device=dev)
        bufs = [(torch.empty(T, INTER, dtype=torch.bfloat16, device=dev),
                 torch.empty(T, 2 * INTER, dtype=torch.bfloat16, device=dev),
                 torch.empty(T, 2 * INTER, dtype=torch.bfloat16, device=dev)) for _ in self.sw13]
        self._mark("router")

        def shared_fwd():   # runs on a side stream while the rows are in flight
            for (h, gu, _), w13, w2 in zip(bufs, self.sw13, self.sw2):
                C.swiglu_fwd(x, w13, self.empty_i32, h, gu)
                C.linear_fwd(h, w2, out, True)

        def shared_bwd():
            for (h, gu, dgu), w13, w2, g13, g2 in zip(bufs, self.sw13, self.sw2, self.sg13, self.sg2):
                C.swiglu_dgrad(self.dout, w2.view(1, D, INTER), self.empty_i32, gu, dgu)
                C.linear_wgrad(self.dout, h, g2)
                C.linear_dgrad(dgu, w13.view(2 * INTER, D), dx, True)
                C.linear_wgrad(dgu, x, g13)
        ctx = moe_forward_ep(self.ep, 0, x, idx, wts, counts, self.w13, self.w2, out, INTER,
                             marks=self._mark, overlap=shared_fwd)
        self.cnt_all = ctx["cnt_all"]
        dw = moe_backward_ep(self.ep, ctx, self.dout, self.w13, self.w2, self.g13, self.g2, dx, INTER,
                             marks=self._mark, overlap=shared_bwd)
        dlog = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
        C.router_bwd(dw, ssel, idx, 1.0, dlog)
        C.linear_wgrad(dlog, x, self.ggate)
        C.linear_dgrad(dlog, self.gate, dx, True)
        self._mark("router bwd")
        return out, dx

    def phases(self):
        """Device ms between consecutive marks of one instrumented step."""
        self.events = []
        self.step()
        torch.cuda.synchronize()
        ev, self.events = self.events, None
        return [(n1, e0.elapsed_time(e1)) for (_, e0), (n1, e1) in zip(ev, ev[1:])]

    def remote_rows(self):
        """(rows this rank sends to others, rows it receives from others) per transfer phase."""
        cnt = self.cnt_all.cpu()
        me, lo, hi = self.ep.rank, self.ep.lo, self.ep.hi
        sent = int(cnt[me].sum()) - int(cnt[me, lo:hi].sum())
        recv = int(cnt[:, lo:hi].sum()) - int(cnt[me, lo:hi].sum())
        return sent, recv

    def close(self):
        self.ep.close()


# ---------------------------------------------------------------- reference
class ReferenceLayer:
    """The reference's gate and expert modules behind an NCCL all-to-all harness."""

    def __init__(self, T: int, rank: int, world: int, device):
        root = HERE.parent.parent / "baseline" / "_ref"
        if not (root / "models" / "moe.py").exists():
            raise FileNotFoundError("reference not installed in baseline/_ref")
        sys.path.insert(0, str(root))
        for m in [m for m in sys.modules if m == "models" or m.startswith("models.")]:
            del sys.modules[m]
        from models.moe import AuxLossFreeGate, Expert  # the reference's own modules
        self.world, self.rank = world, rank
        cfg = {"dim": D, "n_routed_experts": E, "n_activated_experts": TOPK, "route_scale": 1.0}
        torch.manual_seed(0)
        self.gate = AuxLossFreeGate(cfg).to(device)
        with torch.no_grad():
            self.gate.weight.normal_(0, 0.02)
        self.lo, self.hi = rank * E // world, (rank + 1) * E // world
        self.experts = torch.nn.ModuleList([Expert(D, INTER) for _ in range(self.hi - self.lo)]).to(device)
        self.shared = torch.nn.ModuleList([Expert(D, INTER) for _ in range(N_SHARED)]).to(device)
        self.owner = torch.tensor([next(d for d in range(world - 1, -1, -1) if d * E // world <= e)
                                   for e in range(E)], device=device)
        g = torch.Generator(device="cpu").manual_seed(100 + rank)
        self.x = torch.randn(T, D, generator=g).to(device)
        self.dout = (torch.randn(T, D, generator=g) * 0.01).to(device)
        self.T = T

    def step(self):
        import torch.distributed as dist
        import torch.distributed.nn.functional as dfn
        x = self.x.detach().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            w, idx = self.gate(x)
            flat = idx.reshape(-1)
            order = torch.argsort(self.owner[flat] * E + flat)
            tok = order // TOPK
            dest = self.owner[flat[order]]
            send = torch.bincount(dest, minlength=self.world)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send)
            send_l, recv_l = send.tolist(), recv.tolist()
            rows = x[tok].to(torch.bfloat16)
            got = dfn.all_to_all_single(torch.empty(sum(recv_l), D, device=x.device, dtype=rows.dtype), rows,
                                        recv_l, send_l)
            ids = torch.empty(sum(recv_l), dtype=flat.dtype, device=x.device)
            dist.all_to_all_single(ids, flat[order].contiguous(), recv_l, send_l)
            outs = torch.zeros_like(got)
            for e in range(self.lo, self.hi):
                sel = (ids == e).nonzero(as_tuple=True)[0]
                if sel.numel():
                    outs = outs.index_put((sel,), self.experts[e - self.lo](got[sel]).to(outs.dtype))
            back = dfn.all_to_all_single(torch.empty(sum(send_l), D, device=x.device, dtype=outs.dtype), outs,
                                         send_l, recv_l)
            y = torch.zeros(self.T, D, device=x.device, dtype=torch.float32)
            y = y.index_add(0, tok, back.float() * w.reshape(-1)[order].float().unsqueeze(1))
            for s in self.shared:
                y = y + s(x).float()
        y.backward(self.dout)
        return y, x.grad

    def close(self):
        pass


def run(impl: str, tokens_list, warmup: int, iters: int):
    import torch.distributed as dist
    sys.path.insert(0, str(HERE.parent))
    from parallel.dist import init_distributed
    rank, world, device = init_distributed(timeout_s=120)
    peak_tf, _, peak_src = _peaks()
    rows = []
    for T in tokens_list:
        layer = (OursLayer if impl == "ours" else ReferenceLayer)(T, rank, world, device)
        ms = _max_over_ranks(_time(layer.step, warmup, iters))
        r = {"tokens_per_rank": T, "layer_fwd_bwd_ms": round(ms, 3),
             "tokens_per_s": round(world * T / (ms / 1e3), 1),
             "tflops_per_gpu": round(_flops(T) / (ms / 1e3) / 1e12, 1)}
        if impl == "ours":
            ph = layer.phases()
            sent, recv = layer.remote_rows()
            bytes_phase = max(_max_over_ranks(sent), _max_over_ranks(recv)) * D * 2
            t_comm = 4 * bytes_phase / (NVLINK_GBS * 1e9) * 1e3
            t_comp = _flops(T) / (peak_tf * 1e12) * 1e3
            r["nvlink_bytes_per_rank_per_phase"] = int(bytes_phase)
            r["roofline_ms"] = round(max(t_comp, t_comm), 3)
            r["roofline_bound"] = "compute" if t_comp >= t_comm else "nvlink"
            r["frac_of_roofline"] = round(max(t_comp, t_comm) / ms, 3)
            phases = {}
            for name, t in ph:
                phases[name] = round(_max_over_ranks(t), 3)
            r["phase_ms_max_over_ranks"] = phases
            comm = {k: v for k, v in phases.items() if k.startswith(("dispatch", "combine"))}
            if bytes_phase > 0:
                r["transfer_frac_of_nvlink_roofline"] = {
                    k: round(bytes_phase / (NVLINK_GBS * 1e9) * 1e3 / v, 3) for k, v in comm.items() if v > 0}
        layer.close()
        del layer
        torch.cuda.empty_cache()
        rows.append(r)
    out = {"metric": "MoE layer fwd+bwd under expert parallelism (device ms, max over ranks)", "impl": impl,
           "ep": world, "layer": f"D{D} E{E}x{INTER} top{TOPK} +{N_SHARED} shared, bf16",
           "peak_bf16_tflops": peak_tf, "peak_source": peak_src, "nvlink_gbs": NVLINK_GBS, "results": rows}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, nargs="+", default=[16384])
    ap.add_argument("--sweep", action="store_true", help="tokens per rank 1K, 2K, ..., 32K")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    toks = [1024 << i for i in range(6)] if a.sweep else a.tokens
    run(a.impl, toks, a.warmup, a.iters)


if __name__ == "__main__":
    main()
