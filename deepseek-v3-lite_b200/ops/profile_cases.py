"""Small, self-contained kernel cases for Nsight Compute captures.

``python -m ops.profile_cases <case>`` (run from ``deepseek-v3-lite_b200/``)
launches each kernel of one case twice on realistic shapes of the 412M
training step and exits; the second launch is the one to capture, e.g.::

    python -m ops.profile_cases swiglu_dgrad && \\
    ncu --set full --clock-control none -k regex:gemm_sm100 -s 1 -c 1 -o prof \\
        python -m ops.profile_cases swiglu_dgrad

``train_step`` runs one full 412M micro-step (16 x 2048 tokens) between
``cudaProfilerStart`` / ``cudaProfilerStop`` for a launch list
(``ncu --metrics gpu__time_duration.sum --profile-from-start off``).
Every case keeps well under a few GB on the device.
"""
from __future__ import annotations

import sys

import torch

from ._ext import native


def _bf(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


def case_gemm_dense():
    C = native()
    a, w = _bf(16384, 768), _bf(2304, 768)
    out = torch.empty(16384, 2304, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        C.linear_fwd(a, w, out)


def case_swiglu_dgrad():
    C = native()
    E, D, I = 20, 768, 384
    rows = [16384 * 4 // E // 256 * 256] * E
    tiles = [e for e, r in enumerate(rows) for _ in range(r // 128)]
    P = sum(rows)
    tg = torch.tensor(tiles, dtype=torch.int32, device="cuda")
    dy, w2, gu = _bf(P, D), _bf(E, D, I), _bf(P, 2 * I)
    dgu = torch.empty_like(gu)
    for _ in range(2):
        C.swiglu_dgrad(dy, w2, tg, gu, dgu, group_rows=256)


def case_dense_dgrad_f32():
    C = native()
    dy, w = _bf(16384, 1080), _bf(1080, 768)
    out = torch.empty(16384, 768, device="cuda")
    for _ in range(2):
        C.linear_dgrad(dy, w, out, False)


def case_resid_fwd():
    """Dense forward with the fp32 residual add (the o-projection shape: 32K x 768 x 768)."""
    C = native()
    a, w = _bf(32768, 768), _bf(768, 768)
    resid = torch.randn(32768, 768, device="cuda")
    out = torch.empty(32768, 768, device="cuda")
    for _ in range(2):
        C.linear_fwd(a, w, out, True, resid)


def _attn_inputs(B=2, H=12, S=2048, DP=80, DV=64):
    Q, K, V = _bf(B * H, S, DP), _bf(B * H, S, DP), _bf(B * H, S, DV)
    O = torch.empty(B, S, H, DV, device="cuda", dtype=torch.bfloat16)
    L = torch.empty(B * H, S, device="cuda")
    return B, H, S, DP, DV, Q, K, V, O, L


def case_fa_fwd_tc():
    C = native()
    B, H, S, DP, DV, Q, K, V, O, L = _attn_inputs()
    for _ in range(2):
        C.flash_fwd_tc(Q, K, V, O, L, 0, 0.1, True, H)


def case_fa_fwd():
    C = native()
    B, H, S, DP, DV, Q, K, V, O, L = _attn_inputs()
    for _ in range(2):
        C.flash_fwd(Q, K, V, O, L, 0, 0.1, True, H)


def case_fa_bwd():
    C = native()
    B, H, S, DP, DV, Q, K, V, O, L = _attn_inputs()
    C.flash_fwd(Q, K, V, O, L, 0, 0.1, True, H)
    dQ = torch.zeros(B * H, S, DP, device="cuda")
    dK, dV = torch.empty_like(dQ), torch.empty(B * H, S, DV, device="cuda")
    delta = torch.empty(B * H, S, device="cuda")
    for _ in range(2):
        C.flash_bwd(Q, K, V, O, O, L, delta, dQ, dK, dV, 0, 0.1, True, H)


def case_fa_bwd_wide():
    """The two-kernel tcgen05 backward on the 412M case above and on the
    DeepSeek-V3 head dims (qk 192, v 128; B2 H16 S2048)."""
    C = native()
    for dims in ({}, {"B": 2, "H": 16, "S": 2048, "DP": 192, "DV": 128}):
        B, H, S, DP, DV, Q, K, V, O, L = _attn_inputs(**dims)
        C.flash_fwd(Q, K, V, O, L, 0, 0.1, True, H)
        dQ = torch.zeros(B * H, S, DP, device="cuda")
        dK, dV = torch.empty_like(dQ), torch.empty(B * H, S, DV, device="cuda")
        delta = torch.empty(B * H, S, device="cuda")
        for _ in range(2):
            C.flash_bwd_wide(Q, K, V, O, O, L, delta, dQ, dK, dV, 0, 0.1, True, H)


def _ce_inputs(T=16384, V=100018, D=768):
    x, w = _bf(T, D), _bf(V, D) * 0.05
    tgt = torch.randint(0, V, (T,), device="cuda")
    return T, V, D, x, w, tgt


def case_ce_fwd():
    """Fused LM head + log-sum-exp partials, 16K rows x 100,018 vocab x 768."""
    C = native()
    T, V, D, x, w, tgt = _ce_inputs()
    nt = (V + 255) // 256
    pmax = torch.empty(T, 2 * nt, device="cuda")
    psum = torch.empty(T, 2 * nt, device="cuda")
    tl = torch.zeros(T, device="cuda")
    for _ in range(2):
        C.ce_fwd_partials(x, w, tgt, pmax, psum, tl)


def case_ce_bwd():
    """LM head + cross-entropy gradient epilogue (bf16 dlogits), same shape."""
    C = native()
    T, V, D, x, w, tgt = _ce_inputs()
    lse = torch.full((T,), 12.0, device="cuda")
    scale = torch.full((T,), 1.0 / T, device="cuda")
    dl = torch.empty(T, (V + 63) // 64 * 64, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        C.ce_bwd_logits(x, w, tgt, lse, scale, dl)


def case_latent_decode():
    """Warp-level (mma.sync) absorbed decode: 64 rows x 16 heads over a 4096-row latent cache (R 512 + rope 64)."""
    C = native()
    prev = C.decode_tc(0)
    try:
        _decode_case(C)
    finally:
        C.decode_tc(prev)


def _decode_case(C):
    B, H, R, dr, S = 64, 16, 512, 64, 4096
    q_lat, q_pe = _bf(B, H, R), _bf(B, H, dr)
    kv, pe = _bf(B, S, R), _bf(B, S, dr)
    lens = torch.full((B,), S, dtype=torch.int32, device="cuda")
    scratch = torch.empty(B * H * (S // 256) * (2 + R), device="cuda")
    out = torch.empty(B, H, R, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        C.latent_decode(q_lat, q_pe, kv, pe, lens, 0.07, S, scratch, out)


def case_latent_decode_tc():
    """The same decode case on the tcgen05 kernel (latent_decode_tc.cuh)."""
    C = native()
    prev = C.decode_tc(1)
    try:
        _decode_case(C)
    finally:
        C.decode_tc(prev)


def case_moe_norm_bwd():
    """MoE input gradient fused with the FFN norm backward on the 412M step's
    shapes: 32K tokens, D 768, top-4 of 20 experts, shared-expert part."""
    C = native()
    T, D, E, k = 32768, 768, 20, 4
    P = (T * k + E * 255 + 255) // 256 * 256
    dxs = _bf(P, D)
    dst = torch.randperm(P, device="cuda")[:T * k].view(T, k).int().contiguous()
    dsh = torch.randn(T, D, device="cuda")
    dlog = _bf(T, 24)
    wg = _bf(E, D)
    x = torch.randn(T, D, device="cuda")
    w = torch.ones(D, device="cuda")
    rstd = torch.ones(T, device="cuda")
    dres = torch.zeros(T, D, device="cuda")
    dres_b = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(D, device="cuda")
    for _ in range(2):
        C.moe_norm_bwd(dxs, dst, dsh, dlog, wg, x, w, rstd, dres, dres_b, dw)


def case_ep_dispatch():
    """Expert-parallel dispatch kernel on one rank (the rank stores into its own
    heap): 32K tokens x top-4 of 20 experts, D 768."""
    from parallel.ep import ExpertParallel
    C = native()
    T, E, k, D = 32768, 20, 4, 768
    ep = ExpertParallel(E, k, D, T, n_slots=1)
    x = _bf(T, D)
    logits = torch.randn(T, 24, device="cuda")
    idx = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, device="cuda")
    ssel = torch.empty(T, k, device="cuda")
    for _ in range(2):
        counts = torch.zeros(E, dtype=torch.int32, device="cuda")
        C.router_topk(logits, torch.zeros(E, device="cuda"), E, k, 1.0, idx, w, ssel, counts)
        ep.dispatch(0, x, idx, w, counts)
    torch.cuda.synchronize()
    ep.close()


def case_small_kernels():
    """Every memory-bound kernel of the 412M micro-step once more, on its real
    shapes (32K tokens, D 768, 20 experts top-4, vocab 100,018): router top-k,
    permutation, gather, combine forward / backward, un-permute, router
    backward, RMSNorm forward / backward, embedding forward / backward, MLA
    pack / unpack, CE row / reduce, gradient norm, fused AdamW over a 64M
    flat buffer, and the data-parallel step's kernels on a one-rank
    symmetric heap (barrier, reduce-scatter, norm exchange, update +
    all-gather).  Each runs twice; capture the second."""
    from parallel.dp import FusedDataParallel
    from .rope import rope_cos_sin
    C = native()
    T, D, E, k, V = 32768, 768, 20, 4, 100018
    Ep = 24
    H, dn, dr, dv, R, S, B = 12, 48, 24, 64, 192, 2048, 16
    dev = "cuda"
    f32 = dict(device=dev, dtype=torch.float32)
    i32 = dict(device=dev, dtype=torch.int32)
    logits = torch.randn(T, Ep, **f32)
    bias = torch.zeros(E, **f32)
    idx, wts, ssel = torch.empty(T, k, **i32), torch.empty(T, k, **f32), torch.empty(T, k, **f32)
    P = (T * k + E * 255 + 255) // 256 * 256
    row_off, tg = torch.empty(E + 1, **i32), torch.empty(P // 128, **i32)
    cursor, src, dst = torch.empty(E, **i32), torch.empty(P, **i32), torch.empty(T, k, **i32)
    xn, xs, ys = _bf(T, D), torch.empty(P, D, device=dev, dtype=torch.bfloat16), _bf(P, D)
    out, dacc = torch.zeros(T, D, **f32), torch.zeros(T, D, **f32)
    dres_b, dys, dw = _bf(T, D), torch.empty(P, D, device=dev, dtype=torch.bfloat16), torch.empty(T, k, **f32)
    dlog = torch.empty(T, Ep, device=dev, dtype=torch.bfloat16)
    x, dy = torch.randn(T, D, **f32), torch.randn(T, D, **f32)
    wn, gwn = torch.ones(D, **f32), torch.zeros(D, **f32)
    yb, rs = torch.empty(T, D, device=dev, dtype=torch.bfloat16), torch.empty(T, **f32)
    tok = torch.randint(0, V, (T,), device=dev)
    emb, gemb = torch.randn(V, D, **f32) * 0.01, torch.zeros(V, D, **f32)
    cos, sin = rope_cos_sin(S, dr, 10000.0, torch.device(dev))
    q, kvb, kva = _bf(T, H * (dn + dr)), _bf(T, H * (dn + dv)), _bf(T, R + dr)
    DP = 80
    Qp, Kp = torch.empty(B * H, S, DP, device=dev, dtype=torch.bfloat16), torch.empty(B * H, S, DP, device=dev,
                                                                                    dtype=torch.bfloat16)
    Vt = torch.empty(B * H, S, dv, device=dev, dtype=torch.bfloat16)
    dQ, dK, dV = torch.randn(B * H, S, DP, **f32), torch.randn(B * H, S, DP, **f32), torch.randn(B * H, S, dv, **f32)
    dq, dkvb = torch.empty_like(q), torch.empty_like(kvb)
    dkva = torch.empty(T, R + dr, device=dev, dtype=torch.bfloat16)
    Tt, nt = 2 * T, (V + 255) // 256
    pmax, psum = torch.randn(Tt, 2 * nt, **f32), torch.rand(Tt, 2 * nt, **f32) + 1
    tl, allt = torch.randn(Tt, **f32), torch.randint(0, V, (Tt,), device=dev)
    lse, lrows, rsc = torch.empty(Tt, **f32), torch.empty(Tt, **f32), torch.empty(Tt, **f32)
    seg, segw, losses = torch.tensor([0, T, Tt], **i32), torch.tensor([1.0, 0.3], **f32), torch.empty(2, **f32)
    n = 64 * 1024 * 1024
    master, grad = torch.randn(n, **f32), torch.randn(n, **f32) * 1e-3
    m1, v1, shadow = torch.zeros(n, **f32), torch.zeros(n, **f32), torch.empty(n, device=dev, dtype=torch.bfloat16)
    coef, sq, nrm, scr = torch.ones(1, **f32), torch.zeros(1, **f32), torch.zeros(1, **f32), torch.empty(4096, **f32)
    heap, alloc = FusedDataParallel.make_heap([n])
    hm, hg, hs = alloc("master", n, torch.float32), alloc("grad", n, torch.float32), alloc("shadow", n, torch.bfloat16)
    hm.copy_(master)
    hg.copy_(grad)
    offs = [heap.dp_offs[0], heap.dp_offs[1]]
    om, og, osd = heap.dp_offs[2], heap.dp_offs[3], heap.dp_offs[4]
    expect = torch.zeros(32, **i32)
    budget = int(5e9)
    for it in range(2):
        counts = torch.zeros(E, **i32)
        C.router_topk(logits, bias, E, k, 1.0, idx, wts, ssel, counts)
        C.permute_plan(counts, row_off, tg, cursor, src)
        C.permute_scatter(idx, row_off, cursor, src, dst)
        C.gather_rows(xn, src, k, xs)
        C.combine_fwd(ys, dst, wts, out)
        C.combine_bwd(dres_b, ys, src, wts, k, dys, dw)
        C.unpermute_bwd(dys, dst, dacc)
        C.router_bwd(dw, ssel, idx, 1.0, dlog)
        C.rmsnorm_fwd(x, wn, 1e-6, yb, rs)
        C.rmsnorm_bwd(dy, x, wn, rs, dacc, None, yb, gwn)
        C.embedding_fwd(tok, emb, x)
        C.embedding_bwd(tok, dy, gemb)
        C.mla_pack(q, kvb, kva[:, R:], Qp, Kp, Vt, B, S, H, dn, dr, dv, cos, sin, 0)
        C.mla_unpack(dQ, dK, dV, dq, dkvb, dkva[:, R:], B, S, H, dn, dr, dv, cos, sin, 0)
        C.ce_rows(pmax, psum, tl, allt, lse, lrows)
        C.ce_reduce(lrows, allt, seg, segw, 1.0 / 16, losses, rsc)
        C.grad_sqsum([grad], scr, sq)
        C.adamw_flat(master, grad, m1, v1, shadow, n, 1e-4, 0.9, 0.95, 1e-8, 0.1, it + 1, coef)
        sq.zero_()
        C.dp_barrier(heap.peers, offs, 0, budget, FusedDataParallel.PH_READY, expect)
        C.dp_reduce(heap.peers, offs, 0, budget, og, 0, n, 1.0, sq)
        C.dp_norm(heap.peers, offs, 0, budget, sq, expect, 1.0, nrm, coef)
        C.dp_update(heap.peers, offs, 0, budget, om, og, osd, m1, v1, 0, n, n, 1e-4, 0.9, 0.95, 1e-8, 0.1, it + 1,
                    coef)
        C.dp_barrier(heap.peers, offs, 0, budget, FusedDataParallel.PH_GATHERED, expect)
    torch.cuda.synchronize()
    heap.close()


def case_train_step():
    import os
    import yaml
    from training.pretrain import Pretrainer, config_from_yaml
    here = os.path.dirname(os.path.abspath(__file__))
    y = yaml.safe_load(open(os.path.join(here, "..", "configs", "pretrain_412m.yaml")))
    cfg = config_from_yaml(y)
    cfg.batch_size, cfg.gradient_accumulation_steps = 16, 1000
    cfg.max_steps, cfg.log_per_component_params, cfg.checkpoint_dir = 10 ** 9, False, "/tmp/dsv3_prof_ckpt"
    tr = Pretrainer(cfg)
    S = y["model"]["max_seq_len"]
    d = torch.randint(0, y["model"]["vocab_size"], (16, S + 1), device="cuda")
    for i in range(2):
        tr.train_step(d[:, :-1], d[:, 1:], i)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    tr.train_step(d[:, :-1], d[:, 1:], 2)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


CASES = {k[5:]: v for k, v in globals().items() if k.startswith("case_")}


def main():
    name = sys.argv[1] if len(sys.argv) > 1 else ""
    if name not in CASES:
        raise SystemExit(f"usage: python -m ops.profile_cases {{{'|'.join(sorted(CASES))}}}")
    torch.manual_seed(0)
    CASES[name]()
    torch.cuda.synchronize()
    code = native().status_read()
    print(f"{name}: ok (status {code})")
    if code:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
