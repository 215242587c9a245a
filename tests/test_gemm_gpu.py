"""tcgen05 GEMM engine vs fp32 PyTorch references (B200 only)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[1, 0], ids=["cta_pairs", "single_cta"])
def C(request):
    """Every GEMM test runs with CTA-pair tiles (cta_group::2, where the
    schedule allows them) and with single-CTA tiles."""
    from ops._ext import native
    m = native()
    m.status_reset()
    prev = m.gemm_pairs(-1)
    m.gemm_pairs(request.param)
    yield m
    m.gemm_pairs(prev)
    assert m.status_read() == 0


def bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


def close(out, ref, rtol=2e-2, atol=2e-2):
    if ref.numel() == 0:
        return
    out, ref = out.float(), ref.float()
    err = (out - ref).abs().max().item()
    tol = atol + rtol * ref.abs().max().item()
    assert err <= tol, f"max err {err} > {tol}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 216, 768), (1000, 864, 768), (129, 104, 192),
                                   (4096, 768, 768)])
def test_linear_fwd(C, M, N, K):
    a, w = bf(M, K, seed=1), bf(N, K, scale=0.05, seed=2)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.linear_fwd(a, w, out)
    close(out, a.float() @ w.float().t())
    acc = torch.randn(M, N, device="cuda")
    ref = acc + a.float() @ w.float().t()
    C.linear_fwd(a, w, acc)
    close(acc, ref, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("M,N,K", [(256, 768, 768), (300, 216, 768), (513, 1344, 192)])
def test_linear_dgrad(C, M, N, K):
    dy, w = bf(M, N, seed=3), bf(N, K, scale=0.05, seed=4)
    out = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    C.linear_dgrad(dy, w, out)
    ref = dy.float() @ w.float()
    close(out, ref)
    # fp32 outputs: plain store and accumulate, in a wider buffer whose
    # padding columns and rows must stay untouched
    buf = torch.full((M + 8, K + 8), 5.0, device="cuda")
    o32 = buf[:M, :K]
    C.linear_dgrad(dy, w, o32, False)
    close(o32, ref, rtol=1e-3, atol=1e-3)
    C.linear_dgrad(dy, w, o32, True)
    close(o32, 2 * ref, rtol=1e-3, atol=1e-3)
    assert (buf[:, K:] == 5.0).all() and (buf[M:] == 5.0).all()


@pytest.mark.parametrize("M,N,K", [(4096, 768, 768), (300, 216, 768), (129, 102, 192), (1000, 768, 1536)])
def test_linear_fwd_f32_store_and_residual(C, M, N, K):
    a, w = bf(M, K, seed=7), bf(N, K, scale=0.05, seed=8)
    ref = a.float() @ w.float().t()
    ld = (N + 7) // 8 * 8 + 8            # row stride a multiple of 8; N = 102 takes the register path
    buf = torch.full((M, ld), 5.0, device="cuda")
    out = buf[:, :N]
    C.linear_fwd(a, w, out, False)
    close(out, ref, rtol=1e-3, atol=1e-3)
    resid = torch.randn(M, ld, device="cuda")[:, :N]
    buf2 = torch.full((M, ld), 5.0, device="cuda")
    out2 = buf2[:, :N]
    C.linear_fwd(a, w, out2, True, resid)
    close(out2, resid + ref, rtol=1e-3, atol=1e-3)
    assert (buf[:, N:] == 5.0).all() and (buf2[:, N:] == 5.0).all()


@pytest.mark.parametrize("M,N,K", [(4096, 768, 768), (1000, 216, 768), (16384, 256, 512)])
def test_linear_wgrad(C, M, N, K):
    dy, x = bf(M, N, seed=5), bf(M, K, seed=6)
    dw = torch.randn(N, K, device="cuda")
    ref = dw + dy.float().t() @ x.float()
    C.linear_wgrad(dy, x, dw)
    close(dw, ref, rtol=1e-3, atol=1e-2)


def _groups(counts, rows=128):
    """Padded expert-sorted layout (ranges multiples of ``rows``): row offsets
    and per-128-row-tile expert ids."""
    pad = [((c + rows - 1) // rows) * rows for c in counts]
    off = [0]
    for p in pad:
        off.append(off[-1] + p)
    tiles = []
    for e, p in enumerate(pad):
        tiles += [e] * (p // 128)
    return off, tiles


@pytest.mark.parametrize("group_rows", [128, 256])
@pytest.mark.parametrize("I,D,counts", [(384, 768, [300, 0, 129, 512]), (128, 256, [64, 200])])
def test_swiglu_grouped(C, I, D, counts, group_rows):
    G = len(counts)
    off, tiles = _groups(counts, group_rows)
    P = off[-1]
    x = bf(P, D, seed=7)
    for e in range(G):  # zero the padding rows like the permutation kernel does
        x[off[e] + counts[e]:off[e + 1]] = 0
    w13 = bf(G, 2, I, D, scale=0.05, seed=8)
    tg = torch.tensor(tiles + [-1, -1], dtype=torch.int32, device="cuda")
    h = torch.empty(P, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(P, 2 * I, device="cuda", dtype=torch.bfloat16)
    C.swiglu_fwd(x, w13, tg, h, gu, group_rows=group_rows)
    for e in range(G):
        rows = slice(off[e], off[e] + counts[e])
        g = x[rows].float() @ w13[e, 0].float().t()
        u = x[rows].float() @ w13[e, 1].float().t()
        close(gu[rows, :I], g)
        close(gu[rows, I:], u)
        close(h[rows], torch.nn.functional.silu(g) * u)
    # down projection, grouped
    w2 = bf(G, D, I, scale=0.05, seed=9)
    y = torch.empty(P, D, device="cuda", dtype=torch.bfloat16)
    C.grouped_fwd(h, w2, tg, y, group_rows=group_rows)
    for e in range(G):
        rows = slice(off[e], off[e] + counts[e])
        close(y[rows], h[rows].float() @ w2[e].float().t())
    # backward: dgu from dy through w2 and the saved gate/up
    dy = bf(P, D, seed=10)
    dgu = torch.empty(P, 2 * I, device="cuda", dtype=torch.bfloat16)
    C.swiglu_dgrad(dy, w2, tg, gu, dgu, group_rows=group_rows)
    for e in range(G):
        rows = slice(off[e], off[e] + counts[e])
        dh = dy[rows].float() @ w2[e].float()
        g, u = gu[rows, :I].float(), gu[rows, I:].float()
        s = torch.sigmoid(g)
        close(dgu[rows, :I], dh * u * s * (1 + g * (1 - s)))
        close(dgu[rows, I:], dh * g * s)
    dx = torch.empty(P, D, device="cuda", dtype=torch.bfloat16)
    C.grouped_dgrad(dgu, w13.view(G, 2 * I, D), tg, dx, group_rows=group_rows)
    for e in range(G):
        rows = slice(off[e], off[e] + counts[e])
        close(dx[rows], dgu[rows].float() @ w13[e].view(2 * I, D).float())
    # per-expert weight gradients
    for e in range(G):   # padded rows must not contribute
        dy[off[e] + counts[e]:off[e + 1]] = 0
    dw2 = torch.zeros(G, D, I, device="cuda")
    C.grouped_wgrad(dy, h, torch.tensor(off, dtype=torch.int32, device="cuda"), dw2)
    for e in range(G):
        rows = slice(off[e], off[e] + counts[e])
        close(dw2[e], dy[rows].float().t() @ h[rows].float(), rtol=1e-3, atol=1e-2)


def test_swiglu_dense(C):
    P, D, I = 777, 512, 1536
    x = bf(P, D, seed=11)
    w13 = bf(1, 2, I, D, scale=0.05, seed=12)
    h = torch.empty(P, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(P, 2 * I, device="cuda", dtype=torch.bfloat16)
    C.swiglu_fwd(x, w13, torch.empty(0, dtype=torch.int32, device="cuda"), h, gu)
    g = x.float() @ w13[0, 0].float().t()
    u = x.float() @ w13[0, 1].float().t()
    close(h, torch.nn.functional.silu(g) * u)


@pytest.mark.parametrize("T,D,V", [(300, 256, 1000), (1000, 768, 5003), (200, 128, 777)])
def test_ce_partials_and_grad(C, T, D, V):
    x, w = bf(T, D, seed=13), bf(V, D, scale=0.1, seed=14)
    tgt = torch.randint(0, V, (T,), device="cuda")
    tgt[5] = -100
    nt = 2 * ((V + 255) // 256)   # two partials per 256-column tile
    pm = torch.empty(T, nt, device="cuda")
    ps = torch.empty(T, nt, device="cuda")
    tl = torch.zeros(T, device="cuda")
    C.ce_fwd_partials(x, w, tgt, pm, ps, tl)
    logits = x.float() @ w.float().t()
    lse = torch.logsumexp(logits, -1)
    m = pm.max(-1).values
    got = m + torch.log((ps * torch.exp(pm - m[:, None])).sum(-1))
    close(got, lse, rtol=1e-4, atol=1e-3)
    ok = tgt >= 0
    close(tl[ok], logits[ok, tgt[ok]], rtol=1e-4, atol=1e-3)
    scale = torch.full((T,), 0.5, device="cuda")
    # a view of a larger buffer: the rows past T and the columns past V rounded
    # up to 8 keep their sentinel; columns V .. V rounded up to 8 may be zeroed
    ldo = (V + 8 + 7) // 8 * 8
    v8 = (V + 7) // 8 * 8
    buf = torch.full((T + 40, ldo), 7.0, device="cuda", dtype=torch.bfloat16)
    dl = buf[:T]
    C.ce_bwd_logits(x, w, tgt, lse.contiguous(), scale, dl)
    ref = torch.softmax(logits, -1)
    ref[ok, tgt[ok]] -= 1.0
    close(dl[:, :V], ref * 0.5, rtol=1e-2, atol=2e-3)
    assert (buf[:, v8:] == 7.0).all() and (buf[T:] == 7.0).all()
    pad = buf[:T, V:v8]
    assert ((pad == 0.0) | (pad == 7.0)).all()
