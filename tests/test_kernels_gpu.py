"""Non-GEMM sm_100a kernels vs fp32 PyTorch references (B200 only)."""
import math
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from ops._ext import native
    m = native()
    m.status_reset()
    yield m
    assert m.status_read() == 0


def close(out, ref, rtol=2e-2, atol=2e-2):
    if ref.numel() == 0:
        return
    out, ref = out.float(), ref.float()
    err = (out - ref).abs().max().item()
    tol = atol + rtol * ref.abs().max().item()
    assert err <= tol, f"max err {err} > {tol}"


def test_rmsnorm(C):
    T, D = 1000, 768
    x = torch.randn(T, D, device="cuda")
    w = torch.rand(D, device="cuda") + 0.5
    y = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    r = torch.empty(T, device="cuda")
    C.rmsnorm_fwd(x, w, 1e-6, y, r)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    ref = F.rms_norm(xr, (D,), wr, 1e-6)
    close(y, ref)
    dy = torch.randn(T, D, device="cuda")
    ref.backward(dy)
    acc = torch.randn(T, D, device="cuda")
    acc0 = acc.clone()
    dw = torch.zeros(D, device="cuda")
    cp = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    C.rmsnorm_bwd(dy, x, w, r, acc, None, cp, dw)
    close(acc - acc0, xr.grad, rtol=1e-3, atol=1e-3)
    close(cp, acc)
    close(dw, wr.grad, rtol=1e-3, atol=1e-2)
    # bf16 input (strided latent slice), store mode
    xb = torch.randn(T, 216, device="cuda").bfloat16()
    lat = xb[:, :192]
    wl = torch.rand(192, device="cuda") + 0.5
    yl = torch.empty(T, 192, device="cuda", dtype=torch.bfloat16)
    rl = torch.empty(T, device="cuda")
    C.rmsnorm_fwd(lat, wl, 1e-6, yl, rl)
    close(yl, F.rms_norm(lat.float(), (192,), wl, 1e-6))
    dyl = torch.randn(T, 192, device="cuda").bfloat16()
    dxl = torch.empty(T, 216, device="cuda", dtype=torch.bfloat16)
    dwl = torch.zeros(192, device="cuda")
    C.rmsnorm_bwd(dyl, lat, wl, rl, None, dxl[:, :192], None, dwl)
    lr = lat.float().requires_grad_(True)
    F.rms_norm(lr, (192,), wl, 1e-6).backward(dyl.float())
    close(dxl[:, :192], lr.grad)


def test_rope_and_inverse(C):
    from ops.rope import rope_cos_sin, rope_table, apply_rope_complex
    T, H, S = 256, 4, 128
    cos, sin = rope_cos_sin(S, 24, 10000.0, "cuda")
    x = torch.randn(T, H, 72, device="cuda").bfloat16()
    y = x.clone()
    C.rope_inplace(y, 48, 12, cos, sin, None, S, 0, False)
    ref = apply_rope_complex(x[:, :, 48:].view(2, S, H, 24), rope_table(S, 24, 10000.0, "cuda")).view(T, H, 24)
    close(y[:, :, 48:], ref)
    assert torch.equal(y[:, :, :48], x[:, :, :48])
    C.rope_inplace(y, 48, 12, cos, sin, None, S, 0, True)
    close(y, x)


@pytest.mark.parametrize("B,S,H,dn,dr,dv", [(2, 128, 4, 48, 24, 64), (1, 200, 2, 16, 16, 16)])
def test_flash_attention_vs_reference(C, B, S, H, dn, dr, dv):
    from ops.rope import rope_cos_sin
    torch.manual_seed(0)
    T = B * S
    DP = ((dn + dr + 15) // 16) * 16
    DP = 32 if DP < 32 else DP
    q = (torch.randn(T, H, dn + dr, device="cuda")).bfloat16()
    kvb = (torch.randn(T, H, dn + dv, device="cuda")).bfloat16()
    kv_a = torch.randn(T, 64 + dr, device="cuda").bfloat16()
    kpe = kv_a[:, 64:]
    cos, sin = rope_cos_sin(S, dr, 10000.0, "cuda")
    Q = torch.empty(B * H, S, DP, device="cuda", dtype=torch.bfloat16)
    K = torch.empty_like(Q)
    V = torch.empty(B * H, S, dv, device="cuda", dtype=torch.bfloat16)
    C.mla_pack(q, kvb, kpe, Q, K, V, B, S, H, dn, dr, dv, cos, sin, 0)
    scale = (dn + dr) ** -0.5
    O = torch.empty(B, S, H, dv, device="cuda", dtype=torch.bfloat16)   # token-major output
    L = torch.empty(B * H, S, device="cuda")
    C.flash_fwd(Q, K, V, O, L, 0, scale, True, H)
    Qr = Q.float().requires_grad_(True)
    Kr = K.float().requires_grad_(True)
    Vr = V.float().requires_grad_(True)
    mask = torch.ones(S, S, device="cuda", dtype=torch.bool).tril()
    att = (Qr @ Kr.transpose(1, 2) * scale).masked_fill(~mask, float("-inf")).softmax(-1)
    ref = att @ Vr
    tok = lambda t: t.view(B, H, S, -1).permute(0, 2, 1, 3)
    close(O, tok(ref), rtol=2e-2, atol=2e-2)
    dO = torch.randn(B, S, H, dv, device="cuda").bfloat16()
    ref.backward(dO.float().permute(0, 2, 1, 3).reshape(B * H, S, dv))
    dQ = torch.zeros(B * H, S, DP, device="cuda")
    dK = torch.empty(B * H, S, DP, device="cuda")
    dV = torch.empty(B * H, S, dv, device="cuda")
    delta = torch.empty(B * H, S, device="cuda")
    C.flash_bwd(Q, K, V, O, dO, L, delta, dQ, dK, dV, 0, scale, True, H)
    close(dV, Vr.grad, rtol=3e-2, atol=3e-2)
    close(dK, Kr.grad, rtol=3e-2, atol=3e-2)
    close(dQ, Qr.grad, rtol=3e-2, atol=3e-2)
    # unpack back to projection-output gradients
    dq = torch.empty_like(q)
    dkvb = torch.empty_like(kvb)
    dkva = torch.zeros_like(kv_a)
    C.mla_unpack(dQ, dK, dV, dq, dkvb, dkva[:, 64:], B, S, H, dn, dr, dv, cos, sin, 0)
    close(dkvb[:, :, dn:], dV.view(B, H, S, dv).permute(0, 2, 1, 3).reshape(T, H, dv))
    close(dq[:, :, :dn], dQ.view(B, H, S, DP).permute(0, 2, 1, 3).reshape(T, H, DP)[:, :, :dn])


def test_latent_decode(C):
    B, H, R, dr, S = 3, 4, 128, 32, 700
    q_lat = torch.randn(B, H, R, device="cuda").bfloat16()
    q_pe = torch.randn(B, H, dr, device="cuda").bfloat16()
    kv = torch.randn(B, S, R, device="cuda").bfloat16()
    pe = torch.randn(B, S, dr, device="cuda").bfloat16()
    lens = torch.tensor([700, 1, 333], device="cuda", dtype=torch.int32)
    scale = 0.1
    scratch = torch.empty(B * H * 3 * (2 + R), device="cuda")
    out = torch.empty(B, H, R, device="cuda", dtype=torch.bfloat16)
    C.latent_decode(q_lat, q_pe, kv, pe, lens, scale, S, scratch, out)
    from ops.decode import latent_decode_attention
    ref = latent_decode_attention(q_lat.cpu().float(), q_pe.cpu().float(), kv.cpu().float(), pe.cpu().float(),
                                  lens.cpu().long(), scale)
    close(out.cpu(), ref)


def _check_permutation(idx, counts, row_off, src, dst, xs, x, k):
    """Every (token, slot) owns one row of its expert's range holding the token's
    row; the rest of each range is zero with src = -1; src and dst invert."""
    E = counts.numel()
    ro, cnt = row_off.cpu(), counts.cpu()
    flat = idx.flatten().long().cpu()
    d = dst.flatten().long().cpu()
    s = src.cpu()
    assert torch.equal(s[d], torch.arange(flat.numel(), dtype=torch.int32))
    for e in range(E):
        mine = d[flat == e]
        assert mine.numel() == cnt[e] and ((mine >= ro[e]) & (mine < ro[e] + cnt[e])).all()
        assert (s[ro[e] + cnt[e]:ro[e + 1]] == -1).all()
        assert (xs[ro[e] + cnt[e]:ro[e + 1]] == 0).all()
    assert torch.equal(xs[dst.flatten().long()], x.repeat_interleave(k, 0))


@pytest.mark.parametrize("T,E,k", [(1000, 20, 4), (777, 40, 6), (300, 8, 1)])
def test_permute_gather_shapes(C, T, E, k):
    D = 384
    idx = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]).int()
    counts = torch.bincount(idx.flatten().long(), minlength=E).int()
    P = ((T * k + E * 255 + 255) // 256) * 256
    row_off = torch.empty(E + 1, device="cuda", dtype=torch.int32)
    tg = torch.empty(P // 128, device="cuda", dtype=torch.int32)
    cursor = torch.empty(E, device="cuda", dtype=torch.int32)
    src = torch.empty(P, device="cuda", dtype=torch.int32)
    dst = torch.empty(T, k, device="cuda", dtype=torch.int32)
    x = torch.randn(T, D, device="cuda").bfloat16()
    xs = torch.full((P, D), 3.0, device="cuda", dtype=torch.bfloat16)
    C.permute_plan(counts, row_off, tg, cursor, src, src_tail_only=True)
    C.permute_gather(idx, counts, row_off, cursor, x, src, dst, xs)
    torch.cuda.synchronize()
    _check_permutation(idx, counts, row_off, src, dst, xs, x, k)
    assert (src[row_off[E].item():] == -1).all()



@pytest.mark.parametrize("B,H,R,dr,S,cache_rows,qpb", [
    (64, 16, 512, 64, 700, 700, 1),     # MLA microbenchmark dims (tcgen05 kernel, R 512)
    (5, 12, 192, 24, 1000, 1024, 1),    # 412M dims: 12 heads, rope 24, a cache longer than max_len
    (3, 20, 128, 32, 300, 300, 1),      # two head groups, the second partly empty
    (6, 16, 64, 16, 129, 129, 3),       # three query rows per cache row (speculative verification)
])
@pytest.mark.parametrize("tc", [1, 0], ids=["tcgen05", "mma_sync"])
def test_latent_decode_shapes(C, B, H, R, dr, S, cache_rows, qpb, tc):
    """Absorbed decode against fp32 over each row's own cache length (0, 1,
    tile-straddling and full lengths), on the tcgen05 and the mma.sync kernels."""
    prev = C.decode_tc(tc)
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + R)
    rnd = lambda *sh: torch.randn(*sh, device="cuda", generator=g)
    Bc = B // qpb
    q_lat, q_pe = rnd(B, H, R).bfloat16(), rnd(B, H, dr).bfloat16()
    kv, pe = rnd(Bc, cache_rows, R).bfloat16(), rnd(Bc, cache_rows, dr).bfloat16()
    lens = torch.randint(1, S + 1, (B,), device="cuda", generator=g).int()
    lens[0] = S
    if B > 2:
        lens[1] = 0
        lens[2] = min(S, 129)
    scale = 0.08
    nsplit = (S + 255) // 256
    scratch = torch.empty(B * H * nsplit * (2 + R), device="cuda")
    out = torch.full((B, H, R), float("nan"), device="cuda", dtype=torch.bfloat16)
    try:
        C.latent_decode(q_lat, q_pe, kv, pe, lens, scale, S, scratch, out, qpb)
        torch.cuda.synchronize()
    finally:
        C.decode_tc(prev)
    assert C.status_read() == 0
    ref = torch.zeros(B, H, R, device="cuda")
    for b in range(B):
        n = int(lens[b])
        if n:
            k, p = kv[b // qpb, :n].float(), pe[b // qpb, :n].float()
            ref[b] = torch.softmax((q_lat[b].float() @ k.T + q_pe[b].float() @ p.T) * scale, -1) @ k
    close(out, ref)


def test_router_and_permutation(C):
    T, E, k, D = 1000, 20, 4, 256
    logits = torch.randn(T, 24, device="cuda")
    bias = torch.randn(E, device="cuda") * 0.01
    idx = torch.empty(T, k, device="cuda", dtype=torch.int32)
    w = torch.empty(T, k, device="cuda")
    ssel = torch.empty(T, k, device="cuda")
    counts = torch.zeros(E, device="cuda", dtype=torch.int32)
    C.router_topk(logits, bias, E, k, 1.0, idx, w, ssel, counts)
    s = torch.sigmoid(logits[:, :E])
    ref_idx = torch.topk(s + bias, k, -1).indices
    assert torch.equal(idx.long().sort(-1).values, ref_idx.sort(-1).values)
    picked = s.gather(1, idx.long())
    close(w, picked / picked.sum(-1, keepdim=True), rtol=1e-5, atol=1e-6)
    assert torch.equal(counts.long(), torch.bincount(idx.flatten().long(), minlength=E))
    # permutation
    P = ((T * k + E * 255 + 255) // 256) * 256
    row_off = torch.empty(E + 1, device="cuda", dtype=torch.int32)
    tg = torch.empty(P // 128, device="cuda", dtype=torch.int32)
    cursor = torch.empty(E, device="cuda", dtype=torch.int32)
    src = torch.empty(P, device="cuda", dtype=torch.int32)
    dst = torch.empty(T, k, device="cuda", dtype=torch.int32)
    C.permute_plan(counts, row_off, tg, cursor, src)
    C.permute_scatter(idx, row_off, cursor, src, dst)
    ro = row_off.cpu()
    for e in range(E):
        rows = src[ro[e]:ro[e] + counts[e]].cpu()
        assert (rows >= 0).all() and (idx.flatten().cpu()[rows] == e).all()
        assert (src[ro[e] + counts[e]:ro[e + 1]].cpu() == -1).all()
    x = torch.randn(T, D, device="cuda").bfloat16()
    xs = torch.empty(P, D, device="cuda", dtype=torch.bfloat16)
    C.gather_rows(x, src, k, xs)
    assert torch.equal(xs[dst.flatten().long()], x.repeat_interleave(k, 0))
    # the fused permutation + gather gives the same ranges, rows and padding
    xs2 = torch.full((P, D), 7.0, device="cuda", dtype=torch.bfloat16)
    src2 = torch.empty(P, device="cuda", dtype=torch.int32)
    dst2 = torch.empty(T, k, device="cuda", dtype=torch.int32)
    C.permute_plan(counts, row_off, tg, cursor, src2, src_tail_only=True)
    C.permute_gather(idx, counts, row_off, cursor, x, src2, dst2, xs2)
    _check_permutation(idx, counts, row_off, src2, dst2, xs2, x, k)
    # combine forward / backward
    y = torch.randn(P, D, device="cuda").bfloat16()
    out = torch.zeros(T, D, device="cuda")
    C.combine_fwd(y, dst, w, out)
    ref = (y[dst.long()].float() * w[..., None]).sum(1)
    close(out, ref, rtol=1e-3, atol=1e-3)
    dout = torch.randn(T, D, device="cuda").bfloat16()
    dy = torch.empty(P, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(T, k, device="cuda")
    C.combine_bwd(dout, y, src, w, k, dy, dw)
    close(dy[dst.long()], dout.float()[:, None] * w[..., None])
    close(dw, (dout.float()[:, None] * y[dst.long()].float()).sum(-1), rtol=1e-3, atol=1e-2)
    pad = src < 0
    assert (dy[pad] == 0).all()
    # unpermute + router backward
    acc = torch.zeros(T, D, device="cuda")
    C.unpermute_bwd(dy, dst, acc)
    close(acc, dy[dst.long()].float().sum(1), rtol=1e-3, atol=1e-3)
    dl = torch.empty(T, 24, device="cuda", dtype=torch.bfloat16)
    C.router_bwd(dw, ssel, idx, 1.0, dl)
    lr = logits[:, :E].clone().requires_grad_(True)
    sr = torch.sigmoid(lr)
    pk = sr.gather(1, idx.long())
    (pk / pk.sum(-1, keepdim=True) * dw).sum().backward()
    close(dl[:, :E], lr.grad, rtol=2e-2, atol=1e-3)
    assert (dl[:, E:] == 0).all()


def test_adamw_and_norm(C):
    n = 100003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda") * 3
    ref_p = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref_p], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    scratch = torch.empty(4096, device="cuda")
    sq = torch.empty(1, device="cuda")
    C.grad_sqsum([g], scratch, sq)
    close(sq, (g.double() ** 2).sum().float(), rtol=1e-5, atol=0)
    norm = torch.empty(1, device="cuda")
    coef = torch.empty(1, device="cuda")
    C.clip_coef(sq, 1.0, norm, coef)
    for step in (1, 2, 3):
        ref_p.grad = g * coef
        opt.step()
        C.adamw_flat(p, g, m, v, sh, n, 1e-2, 0.9, 0.95, 1e-8, 0.1, step, coef)
    close(p, ref_p.detach(), rtol=1e-5, atol=1e-6)
    close(sh, p)


def test_embedding(C):
    V, D, T = 1000, 256, 300
    w = torch.randn(V, D, device="cuda")
    tok = torch.randint(0, V, (T,), device="cuda")
    out = torch.empty(T, D, device="cuda")
    C.embedding_fwd(tok, w, out)
    assert torch.equal(out, w[tok])
    g = torch.randn(T, D, device="cuda")
    dw = torch.zeros(V, D, device="cuda")
    C.embedding_bwd(tok, g, dw)
    ref = torch.zeros(V, D, device="cuda").index_add_(0, tok, g)
    close(dw, ref, rtol=1e-5, atol=1e-5)


def test_embedding_rejects_out_of_range_ids(C):
    """An id outside [0, V) is never dereferenced: its row reads as zeros, its
    gradient is dropped and the status word reports a bounds error."""
    V, D = 100, 64
    w = torch.randn(V, D, device="cuda")
    tok = torch.tensor([3, V, -1, 7], device="cuda")
    out = torch.full((4, D), 9.0, device="cuda")
    C.status_reset()
    C.embedding_fwd(tok, w, out)
    assert C.status_read() == 5
    assert torch.equal(out[0], w[3]) and torch.equal(out[3], w[7])
    assert out[1].abs().sum().item() == 0 and out[2].abs().sum().item() == 0
    C.status_reset()
    dw = torch.zeros(V, D, device="cuda")
    C.embedding_bwd(tok, torch.ones(4, D, device="cuda"), dw)
    assert C.status_read() == 5
    assert dw.sum().item() == 2 * D
    C.status_reset()


def test_ce_finalize(C):
    T, V = 300, 1000
    x = torch.randn(T, 256, device="cuda").bfloat16()
    w = (torch.randn(V, 256, device="cuda") * 0.1).bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    tgt[:7] = -100
    nt = 2 * ((V + 255) // 256)   # two partials per 256-column tile
    pm, ps = torch.empty(T, nt, device="cuda"), torch.empty(T, nt, device="cuda")
    tl = torch.zeros(T, device="cuda")
    C.ce_fwd_partials(x, w, tgt, pm, ps, tl)
    lse, lrows = torch.empty(T, device="cuda"), torch.empty(T, device="cuda")
    C.ce_rows(pm, ps, tl, tgt, lse, lrows)
    seg = torch.tensor([0, 200, 300], device="cuda", dtype=torch.int32)
    segw = torch.tensor([1.0, 0.3], device="cuda")
    loss = torch.empty(2, device="cuda")
    rsc = torch.empty(T, device="cuda")
    C.ce_reduce(lrows, tgt, seg, segw, 0.5, loss, rsc)
    logits = x.float() @ w.float().t()
    ref0 = F.cross_entropy(logits[:200], tgt[:200], ignore_index=-100)
    ref1 = F.cross_entropy(logits[200:], tgt[200:], ignore_index=-100)
    close(loss, torch.stack([ref0, ref1]), rtol=1e-4, atol=1e-4)
    assert rsc[0].item() == 0 and abs(rsc[10].item() - 0.5 / 193) < 1e-7


def _attn_ref(Q, K, V, scale, causal, q_off=0):
    s = Q.float() @ K.float().transpose(1, 2) * scale
    if causal:
        sq, sk = Q.shape[1], K.shape[1]
        qi = torch.arange(sq, device=Q.device)[:, None] + q_off
        ki = torch.arange(sk, device=Q.device)[None, :]
        s = s.masked_fill(ki > qi, float("-inf"))
    return s.softmax(-1) @ V.float()


@pytest.mark.parametrize("B,H,S,DP,DV", [(2, 3, 2048, 80, 64), (1, 2, 300, 80, 64), (2, 2, 1000, 64, 64),
                                         (1, 2, 640, 128, 128), (1, 2, 700, 192, 128)])
def test_flash_fwd_tcgen05(C, B, H, S, DP, DV):
    torch.manual_seed(0)
    Q = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    K = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    V = torch.randn(B * H, S, DV, device="cuda").bfloat16()
    if DP == 80:
        Q[..., 72:] = 0
        K[..., 72:] = 0
    scale = 0.11
    O = torch.empty(B, S, H, DV, device="cuda", dtype=torch.bfloat16)
    L = torch.empty(B * H, S, device="cuda")
    C.flash_fwd_tc(Q, K, V, O, L, 0, scale, True, H)
    ref = _attn_ref(Q, K, V, scale, True).view(B, H, S, DV).permute(0, 2, 1, 3)
    close(O, ref, rtol=2e-2, atol=2e-2)
    # log-sum-exp (log2 domain) agrees with the warp-level kernel
    O2 = torch.empty_like(O)
    L2 = torch.empty_like(L)
    C.flash_fwd_mma(Q, K, V, O2, L2, 0, scale, True, H)
    close(L, L2, rtol=1e-3, atol=1e-2)
    close(O, O2, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("B,H,S,DP,DV", [(2, 3, 2048, 80, 64), (1, 2, 300, 80, 64), (2, 2, 1000, 64, 64)])
def test_flash_bwd_tcgen05(C, B, H, S, DP, DV):
    torch.manual_seed(1)
    Q = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    K = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    V = torch.randn(B * H, S, DV, device="cuda").bfloat16()
    if DP == 80:
        Q[..., 72:] = 0
        K[..., 72:] = 0
    scale = 0.11
    O = torch.empty(B, S, H, DV, device="cuda", dtype=torch.bfloat16)
    L = torch.empty(B * H, S, device="cuda")
    C.flash_fwd(Q, K, V, O, L, 0, scale, True, H)
    dO = torch.randn(B, S, H, DV, device="cuda").bfloat16()
    grads = []
    for fn in (C.flash_bwd, C.flash_bwd_mma):
        dQ = torch.zeros(B * H, S, DP, device="cuda")
        dK = torch.empty(B * H, S, DP, device="cuda")
        dV = torch.empty(B * H, S, DV, device="cuda")
        delta = torch.empty(B * H, S, device="cuda")
        fn(Q, K, V, O, dO, L, delta, dQ, dK, dV, 0, scale, True, H)
        grads.append((dQ, dK, dV))
    Qr, Kr, Vr = (t.float().requires_grad_(True) for t in (Q, K, V))
    ref = _attn_ref(Qr, Kr, Vr, scale, True)
    ref.backward(dO.float().permute(0, 2, 1, 3).reshape(B * H, S, DV))
    for got in grads:
        close(got[2], Vr.grad, rtol=3e-2, atol=3e-2)
        close(got[1], Kr.grad, rtol=3e-2, atol=3e-2)
        close(got[0], Qr.grad, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("B,H,S,DP,DV", [(1, 2, 1000, 192, 128), (2, 2, 512, 128, 128), (1, 1, 300, 192, 128),
                                         (2, 3, 700, 80, 64)])
def test_flash_bwd_wide(C, B, H, S, DP, DV):
    """dQ / dK / dV of the two-kernel tcgen05 backward vs the fp32 PyTorch
    reference and vs the backward flash_bwd selects by default."""
    torch.manual_seed(2)
    Q = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    K = torch.randn(B * H, S, DP, device="cuda").bfloat16()
    V = torch.randn(B * H, S, DV, device="cuda").bfloat16()
    if DP == 80:   # qk 72 padded to 80, as the 412M layers pack it
        Q[..., 72:] = 0
        K[..., 72:] = 0
    scale = DP ** -0.5
    O = torch.empty(B, S, H, DV, device="cuda", dtype=torch.bfloat16)
    L = torch.empty(B * H, S, device="cuda")
    C.flash_fwd(Q, K, V, O, L, 0, scale, True, H)
    dO = torch.randn(B, S, H, DV, device="cuda").bfloat16()
    grads = []
    for fn in (C.flash_bwd_wide, C.flash_bwd):
        dQ = torch.zeros(B * H, S, DP, device="cuda")
        dK = torch.empty(B * H, S, DP, device="cuda")
        dV = torch.empty(B * H, S, DV, device="cuda")
        delta = torch.empty(B * H, S, device="cuda")
        fn(Q, K, V, O, dO, L, delta, dQ, dK, dV, 0, scale, True, H)
        torch.cuda.synchronize()
        assert C.status_read() == 0
        grads.append((dQ, dK, dV))
    Qr, Kr, Vr = (t.float().requires_grad_(True) for t in (Q, K, V))
    ref = _attn_ref(Qr, Kr, Vr, scale, True)
    ref.backward(dO.float().permute(0, 2, 1, 3).reshape(B * H, S, DV))
    for got in grads:
        close(got[2], Vr.grad, rtol=3e-2, atol=3e-2)
        close(got[1], Kr.grad, rtol=3e-2, atol=3e-2)
        close(got[0], Qr.grad, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("D,E,with_shared,with_routed", [(256, 20, True, True), (768, 20, False, True),
                                                        (768, 40, True, False), (128, 6, True, True)])
def test_moe_norm_bwd_fused(C, D, E, with_shared, with_routed):
    """Shared + un-permuted routed + router-logit input gradient, then the
    RMSNorm backward, against an fp32 reference of the same sum."""
    T, k = 333, 4
    P = T * k + 64
    g = torch.Generator(device="cuda").manual_seed(5)
    rnd = lambda *s: torch.randn(*s, device="cuda", generator=g)
    dxs = rnd(P, D).bfloat16()
    dst = torch.randperm(P, device="cuda", generator=g)[:T * k].view(T, k).int().contiguous()
    dsh = rnd(T, D)
    Ep = (E + 7) // 8 * 8
    dlog = rnd(T, Ep).bfloat16()
    wg = (rnd(E, D) * 0.2).bfloat16()
    x = rnd(T, D)
    w = 1.0 + 0.1 * rnd(D)
    rstd = torch.rsqrt(x.pow(2).mean(-1) + 1e-6)
    dres0 = rnd(T, D)
    dres = dres0.clone()
    dres_b = torch.empty(T, D, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(D, device="cuda")
    C.moe_norm_bwd(dxs if with_routed else None, dst if with_routed else None, dsh if with_shared else None,
                   dlog, wg, x, w, rstd, dres, dres_b, dw)
    gsum = dlog[:, :E].float() @ wg.float()
    if with_shared:
        gsum = gsum + dsh
    if with_routed:
        gsum = gsum + dxs.float()[dst.long()].sum(1)
    xh = x * rstd[:, None]
    gw = gsum * w
    d = rstd[:, None] * (gw - xh * (gw * xh).mean(-1, keepdim=True))
    close(dres, dres0 + d, rtol=1e-4, atol=1e-4)
    close(dres_b, dres0 + d, rtol=1e-2, atol=1e-2)
    close(dw, (gsum * xh).sum(0), rtol=1e-4, atol=1e-3)
    assert C.status_read() == 0


@pytest.mark.parametrize("B,S,H,hd,DP,col0", [(2, 150, 3, 64, 64, 0), (2, 150, 3, 64, 80, 192), (1, 77, 2, 20, 32, 48)])
def test_heads_pack_unpack(C, B, S, H, hd, DP, col0):
    """[T, ld] head slices <-> [B*H, S, DP] (zero padded), on the 16-byte path
    and (hd 20) the scalar one."""
    T = B * S
    ld = col0 + H * hd + 8
    src = torch.randn(T, ld, device="cuda").bfloat16()
    dst = torch.full((B * H, S, DP), 3.0, device="cuda", dtype=torch.bfloat16)
    C.heads_pack(src, col0, H, hd, S, dst)
    ref = torch.zeros(B * H, S, DP, device="cuda", dtype=torch.bfloat16)
    ref[:, :, :hd] = src[:, col0:col0 + H * hd].view(B, S, H, hd).permute(0, 2, 1, 3).reshape(B * H, S, hd)
    assert torch.equal(dst, ref)
    g = torch.randn(B * H, S, DP, device="cuda")
    out = torch.full((T, ld), 5.0, device="cuda", dtype=torch.bfloat16)
    C.heads_unpack(g, H, hd, S, out, col0)
    want = g[:, :, :hd].view(B, H, S, hd).permute(0, 2, 1, 3).reshape(T, H * hd).bfloat16()
    assert torch.equal(out[:, col0:col0 + H * hd], want)
    assert (out[:, :col0] == 5.0).all() and (out[:, col0 + H * hd:] == 5.0).all()
