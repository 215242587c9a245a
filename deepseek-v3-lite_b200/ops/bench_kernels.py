"""Kernel microbenchmarks (CUDA-event timing, warm-up, no profiler).

``python -m ops.bench_kernels`` (from ``deepseek-v3-lite_b200/``) prints one
JSON line per case: the tcgen05 GEMM engine on square and training-step
shapes (forward, data gradient, weight gradient; cuBLAS via ``torch.matmul``
on the same forward shape for reference; with and without CTA-pair tiles)
and the attention kernels (tcgen05
vs warp-level mma.sync) on the 412M, MTP and MLA-microbenchmark head dims.
``--wide-bwd`` adds the two-kernel tcgen05 backward (``flash_bwd_wide``);
``--lm-head-only`` times the fused LM head + cross-entropy GEMMs alone.
"""
from __future__ import annotations

import argparse
import json

import torch

from ._ext import native


def _time(fn, iters=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def gemm_cases(C):
    out = []
    for (M, N, K) in [(8192, 8192, 8192), (32768, 1080, 768), (32768, 768, 768), (32768, 2304, 768),
                      (32768, 768, 1536)]:
        a = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        dy = torch.randn(M, N, device="cuda").bfloat16()
        dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        dw = torch.zeros(N, K, device="cuda")
        fl = 2.0 * M * N * K
        f = _time(lambda: C.linear_fwd(a, w, o))
        cb = _time(lambda: torch.matmul(a, w.t(), out=o))
        d = _time(lambda: C.linear_dgrad(dy, w, dx))
        g = _time(lambda: C.linear_wgrad(dy, a, dw))
        out.append({"case": f"gemm {M}x{N}x{K}", "fwd_tflops": round(fl / f / 1e9, 1),
                    "dgrad_tflops": round(fl / d / 1e9, 1), "wgrad_tflops": round(fl / g / 1e9, 1),
                    "cublas_fwd_tflops": round(fl / cb / 1e9, 1)})
    return out


def attention_cases(C, wide_bwd=False):
    out = []
    for (B, H, S, DP, DV, dqk) in [(16, 12, 2048, 80, 64, 72), (16, 12, 2046, 64, 64, 64),
                                   (8, 16, 4096, 128, 128, 128), (8, 16, 4096, 192, 128, 192)]:
        Q = torch.randn(B * H, S, DP, device="cuda").bfloat16()
        K = torch.randn_like(Q)
        V = torch.randn(B * H, S, DV, device="cuda").bfloat16()
        O = torch.empty(B, S, H, DV, device="cuda", dtype=torch.bfloat16)
        L = torch.empty(B * H, S, device="cuda")
        fl = 2.0 * B * H * S * S / 2 * (dqk + DV)   # causal forward FLOPs (useful work)
        r = {"case": f"attention B{B} H{H} S{S} dqk{dqk} dv{DV} causal"}
        r["fwd_tcgen05_tflops"] = round(fl / _time(lambda: C.flash_fwd_tc(Q, K, V, O, L, 0, 0.1, True, H)) / 1e9, 1)
        r["fwd_mma_sync_tflops"] = round(fl / _time(lambda: C.flash_fwd_mma(Q, K, V, O, L, 0, 0.1, True, H)) / 1e9, 1)
        if DP <= 80:
            dQ = torch.zeros(B * H, S, DP, device="cuda")
            dK, dV = torch.empty_like(dQ), torch.empty(B * H, S, DV, device="cuda")
            delta = torch.empty(B * H, S, device="cuda")
            tb = _time(lambda: C.flash_bwd(Q, K, V, O, O, L, delta, dQ, dK, dV, 0, 0.1, True, H), 5)
            tm = _time(lambda: C.flash_bwd_mma(Q, K, V, O, O, L, delta, dQ, dK, dV, 0, 0.1, True, H), 5)
            r["bwd_tcgen05_tflops"] = round(2.5 * fl / tb / 1e9, 1)
            r["bwd_mma_sync_tflops"] = round(2.5 * fl / tm / 1e9, 1)
        if wide_bwd and DP in (80, 128, 192):
            # the two-kernel tcgen05 backward (opt-in until validated); the
            # rate counts the useful 2.5x forward FLOPs, not its recomputation
            dQ = torch.zeros(B * H, S, DP, device="cuda")
            dK, dV = torch.empty_like(dQ), torch.empty(B * H, S, DV, device="cuda")
            delta = torch.empty(B * H, S, device="cuda")
            tw = _time(lambda: C.flash_bwd_wide(Q, K, V, O, O, L, delta, dQ, dK, dV, 0, 0.1, True, H), 5)
            r["bwd_two_kernel_tcgen05_tflops"] = round(2.5 * fl / tw / 1e9, 1)
        out.append(r)
    return out


def lm_head_cases(C, rows=65520, chunk=16380, V=100018, D=768):
    """Fused LM head + cross-entropy on the 412M step's shapes: the forward
    partials over all main + MTP rows, then per row chunk the dlogits epilogue
    GEMM and the two gradient GEMMs that read it.  The 154 MB vocabulary
    weight exceeds L2, so the tile order decides how often it is re-read."""
    x = torch.randn(rows, D, device="cuda").bfloat16()
    w = (torch.randn(V, D, device="cuda") * 0.05).bfloat16()
    tgt = torch.randint(0, V, (rows,), device="cuda")
    nt = (V + 255) // 256
    pm, ps = torch.empty(rows, 2 * nt, device="cuda"), torch.empty(rows, 2 * nt, device="cuda")
    tl = torch.zeros(rows, device="cuda")
    lse = torch.full((rows,), 12.0, device="cuda")
    scale = torch.full((rows,), 1.0 / rows, device="cuda")
    dl = torch.empty(chunk, (V + 63) // 64 * 64, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(V, D, device="cuda")
    dx = torch.empty(chunk, D, device="cuda")
    fl_fwd = 2.0 * rows * V * D
    fl_chunk = 2.0 * chunk * V * D
    t_fwd = _time(lambda: C.ce_fwd_partials(x, w, tgt, pm, ps, tl), 5)
    xc, tc, lc, sc = x[:chunk], tgt[:chunk], lse[:chunk], scale[:chunk]
    t_bwd = _time(lambda: C.ce_bwd_logits(xc, w, tc, lc, sc, dl), 5)
    t_wg = _time(lambda: C.linear_wgrad(dl[:, :V], xc, dw), 5)
    t_dg = _time(lambda: C.linear_dgrad(dl[:, :V], w, dx, False), 5)
    return [{"case": f"lm head + CE, {rows} rows x V {V} x D {D} (bwd chunks of {chunk})",
             "fwd_partials_ms": round(t_fwd, 3), "fwd_tflops": round(fl_fwd / t_fwd / 1e9, 1),
             "bwd_dlogits_ms_per_chunk": round(t_bwd, 3), "bwd_dlogits_tflops": round(fl_chunk / t_bwd / 1e9, 1),
             "wgrad_ms_per_chunk": round(t_wg, 3), "dgrad_ms_per_chunk": round(t_dg, 3)}]


def decode_cases(C):
    """Absorbed latent decode (the MLA microbenchmark's decode: 64 rows x 16
    heads over a 4096-row cache of R 512 + rope 64): cache bytes read per
    step over the kernel time (split + merge)."""
    out = []
    for (B, H, R, dr, S) in [(64, 16, 512, 64, 4096), (64, 12, 192, 24, 2048)]:
        q_lat, q_pe = torch.randn(B, H, R, device="cuda").bfloat16(), torch.randn(B, H, dr, device="cuda").bfloat16()
        kv, pe = torch.randn(B, S, R, device="cuda").bfloat16(), torch.randn(B, S, dr, device="cuda").bfloat16()
        lens = torch.full((B,), S, dtype=torch.int32, device="cuda")
        scratch = torch.empty(B * H * ((S + 255) // 256) * (2 + R), device="cuda")
        o = torch.empty(B, H, R, device="cuda", dtype=torch.bfloat16)
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

        def step():
            flush.zero_()             # the cache does not stay in L2 between steps
            C.latent_decode(q_lat, q_pe, kv, pe, lens, 0.07, S, scratch, o)
        t_all = _time(step, 20)
        t_flush = _time(lambda: flush.zero_(), 20)
        t = max(t_all - t_flush, 1e-6)
        nbytes = B * S * (R + dr) * 2
        out.append({"case": f"latent decode B{B} H{H} R{R} rope{dr} ctx{S}", "us": round(t * 1e3, 1),
                    "cache_GBps": round(nbytes / t / 1e6, 1)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--wide-bwd", action="store_true", help="also time the two-kernel tcgen05 attention backward")
    ap.add_argument("--attention-only", action="store_true")
    ap.add_argument("--decode-only", action="store_true")
    ap.add_argument("--lm-head-only", action="store_true")
    a = ap.parse_args()
    C = native()
    if a.lm_head_only:
        for r in lm_head_cases(C):
            print(json.dumps(r), flush=True)
        return
    if a.decode_only:
        for r in decode_cases(C):
            print(json.dumps(r), flush=True)
        return
    for pairs in (() if a.attention_only else (1, 0)):
        C.gemm_pairs(pairs)
        for r in gemm_cases(C):
            r["cta_pairs"] = bool(pairs)
            print(json.dumps(r), flush=True)
    C.gemm_pairs(1)
    for r in attention_cases(C, wide_bwd=a.wide_bwd):
        print(json.dumps(r), flush=True)
    if C.status_read():
        raise SystemExit("kernel status word set")


if __name__ == "__main__":
    main()
