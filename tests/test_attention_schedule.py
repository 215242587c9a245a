"""CPU check of the tile schedules of the two-kernel tcgen05 attention
backward for wide heads (``csrc/attention_bwd_wide.cuh``), restated in
Python: the dK / dV kernel (128-key tiles walking 64-query sub-tiles from
``qstart``) and the dQ kernel (128-query tiles walking ``n_blocks`` key
tiles) each see every visible (query, key) pair exactly once and no other."""
import pytest
import torch


def _visible(Sq, Sk, q_off, causal):
    q = torch.arange(Sq).unsqueeze(1)
    k = torch.arange(Sk).unsqueeze(0)
    return (k <= q + q_off) if causal else torch.ones(Sq, Sk, dtype=torch.bool)


def _kv_kernel_cover(Sq, Sk, q_off, causal):
    seen = torch.zeros(Sq, Sk, dtype=torch.int32)
    nq = (Sq + 63) // 64
    for n0 in range(0, Sk, 128):
        qstart = max(0, int((n0 - q_off) / 64)) if causal else 0    # C++ division truncates toward zero
        for it in range(max(0, nq - qstart)):
            q0 = (qstart + it) * 64
            q = torch.arange(q0, q0 + 64).unsqueeze(0)              # columns of S^T
            key = torch.arange(n0, n0 + 128).unsqueeze(1)           # rows of S^T
            valid = (q < Sq) & (key < Sk) & ((q >= key - q_off) if causal else True)
            qq, kk = torch.broadcast_tensors(q, key)
            seen[qq[valid], kk[valid]] += 1
    return seen


def _dq_kernel_cover(Sq, Sk, q_off, causal):
    seen = torch.zeros(Sq, Sk, dtype=torch.int32)
    for m0 in range(0, Sq, 128):
        n_blocks = (Sk + 127) // 128
        if causal:
            n_blocks = min(n_blocks, (q_off + m0 + 128 + 127) // 128)
        q = torch.arange(m0, m0 + 128).unsqueeze(1)                  # rows of S
        kmax = torch.minimum(torch.full_like(q, Sk - 1), q + q_off) if causal else torch.full_like(q, Sk - 1)
        for j in range(max(0, n_blocks)):
            key = torch.arange(j * 128, j * 128 + 128).unsqueeze(0)
            valid = (q < Sq) & (key <= kmax)
            qq, kk = torch.broadcast_tensors(q, key)
            seen[qq[valid], kk[valid]] += 1
    return seen


@pytest.mark.parametrize("Sq,Sk,q_off,causal", [(300, 300, 0, True), (1000, 1000, 0, True), (200, 700, 500, True),
                                                (130, 260, 130, True), (257, 131, 0, False), (64, 64, 0, True)])
def test_wide_backward_schedules_cover_each_visible_pair_once(Sq, Sk, q_off, causal):
    want = _visible(Sq, Sk, q_off, causal).to(torch.int32)
    assert torch.equal(_kv_kernel_cover(Sq, Sk, q_off, causal), want)
    assert torch.equal(_dq_kernel_cover(Sq, Sk, q_off, causal), want)
