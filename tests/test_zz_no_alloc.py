"""The allocation-free decode entry point (C symbol) against the torch one.

``dsv3_latent_decode_noalloc`` serves callers that cannot allocate device
memory while they run (captured CUDA graphs replayed by a server, fixed
memory budgets, plain C hosts without a caching allocator); it keeps its
split-K scratch in a fixed device array inside the library.  This test calls
it through its exported C symbol (ctypes) and checks it against the
``latent_decode`` entry point and an fp32 PyTorch oracle, on two calls in a
row, then at exactly the array's size limit with an empty row.  It is collected last so
a run that stops at the first failure has already run every other test.
"""
import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _lib():
    import ops._ext  # noqa: F401  (puts torch's libraries in place first)
    path = glob.glob(os.path.join(HERE, "..", "deepseek-v3-lite_b200", "ops", "_dsv3_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.dsv3_latent_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_longlong] * 2 + \
                  [ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _case(seed, B, H, R, dr, S):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g).to(torch.bfloat16)
    lens = torch.randint(1, S + 1, (B,), device="cuda", generator=g, dtype=torch.int32)
    return mk(B, H, R), mk(B, H, dr), mk(B, S, R), mk(B, S, dr), lens


def _fp32_oracle(q_lat, q_pe, kv, pe, lens, scale):
    """softmax(scale * (q_lat . kv + q_pe . pe)) @ kv over each row's first lens[b] cache rows, in fp32."""
    B, H, R = q_lat.shape
    out = torch.zeros(B, H, R, device="cuda")
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        k, p = kv[b, :n].float(), pe[b, :n].float()
        s = (q_lat[b].float() @ k.T + q_pe[b].float() @ p.T) * scale
        out[b] = torch.softmax(s, -1) @ k
    return out


def _call(fn, q_lat, q_pe, kv, pe, lens, max_len, scale):
    B, H, R = q_lat.shape
    out = torch.full((B, H, R), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = fn(q_lat.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), pe.data_ptr(), lens.data_ptr(), B, H, R,
            q_pe.shape[2], kv.stride(0), pe.stride(0), max_len, scale, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out


def _tol(ref):
    return 2e-2 + 2e-2 * ref.float().abs().max().item()


def test_noalloc_matches_entry_point():
    from ops._ext import native
    C = native()
    fn = _lib()
    # two calls in a row through the C symbol: R 512 / rope 64 and R 192 / rope 24
    # (both sizes run on the tcgen05 kernel)
    for seed, (B, H, R, dr, S) in enumerate([(4, 8, 512, 64, 1000), (2, 16, 192, 24, 300)]):
        q_lat, q_pe, kv, pe, lens = _case(seed, B, H, R, dr, S)
        scale = 0.07
        ref = torch.empty(B, H, R, device="cuda", dtype=torch.bfloat16)
        nsplit = (S + 255) // 256
        scratch = torch.empty(B * H * nsplit * (2 + R), device="cuda")
        C.latent_decode(q_lat, q_pe, kv, pe, lens, scale, S, scratch, ref)
        rc, out = _call(fn, q_lat, q_pe, kv, pe, lens, S, scale)
        assert rc == 0
        # same launcher, same kernels: the two entry points agree to the bit
        assert torch.equal(out, ref)
        oracle = _fp32_oracle(q_lat, q_pe, kv, pe, lens, scale)
        err = (out.float() - oracle).abs().max().item()
        assert err <= _tol(oracle), err


def test_noalloc_at_the_scratch_limit_and_empty_rows():
    fn = _lib()
    # B * H * ceil(max_len / 256) * (R + 2) = 4 * 16 * 256 * 256 = 4 Mi floats, exactly the array
    B, H, R, dr, S = 4, 16, 254, 32, 65536
    q_lat, q_pe, kv, pe, lens = _case(7, B, H, R, dr, S)
    lens[1] = 0                       # an empty row yields zeros
    lens[2] = S                       # a row that uses every split
    scale = 0.05
    rc, out = _call(fn, q_lat, q_pe, kv, pe, lens, S, scale)
    assert rc == 0
    assert torch.count_nonzero(out[1]) == 0
    oracle = _fp32_oracle(q_lat, q_pe, kv, pe, lens, scale)
    err = (out.float() - oracle).abs().max().item()
    assert err <= _tol(oracle), err
    # one split more than the array holds is refused and launches nothing
    rc, out = _call(fn, q_lat, q_pe, kv, pe, lens, S + 1, scale)
    assert rc == 1 and torch.isnan(out.float()).all()


def test_noalloc_rejects_oversize():
    fn = _lib()
    x = torch.zeros(8, device="cuda", dtype=torch.bfloat16)
    lens = torch.ones(1, device="cuda", dtype=torch.int32)
    # 64 * 64 * 16 splits * (1024 + 2) floats is far above the 4 Mi-float array
    rc = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), lens.data_ptr(), 64, 64, 1024, 64, 0, 0,
            4096, 1.0, x.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
