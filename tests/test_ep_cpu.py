"""Host-side logic of expert parallelism (no GPU): expert ownership, receive
capacity and the receive-layout plan that every rank derives from the
all-gathered routing counts."""
import itertools

import pytest
import torch

from parallel.ep import expert_range, owner_of, plan_reference, receive_capacity


@pytest.mark.parametrize("E,R", [(20, 8), (20, 4), (20, 2), (64, 8), (8, 8), (9, 2), (256, 8), (20, 1)])
def test_expert_ranges_partition_the_experts(E, R):
    seen = []
    sizes = [b - a for a, b in (expert_range(r, E, R) for r in range(R))]
    assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1   # balanced, nobody empty (E >= R)
    for r in range(R):
        lo, hi = expert_range(r, E, R)
        seen.extend(range(lo, hi))
        for e in range(lo, hi):
            assert owner_of(e, E, R) == r
    assert seen == list(range(E))


def test_receive_capacity_covers_the_worst_case():
    T, k, E, R = 1024, 4, 20, 8
    cap = receive_capacity(T, k, E, R)
    assert cap % 128 == 0
    # 3 local experts at most; every token of every rank may send 3 rows to one rank
    assert cap >= R * T * 3 + 3 * 255
    capped = receive_capacity(T, k, E, R, capacity_factor=2.0)
    assert capped < cap and capped >= 2 * T * k


def _random_counts(R, E, T, k, seed):
    g = torch.Generator().manual_seed(seed)
    cnt = torch.zeros(R, E, dtype=torch.int32)
    for s in range(R):
        for _ in range(T):
            for e in torch.randperm(E, generator=g)[:k]:
                cnt[s, e] += 1
    return cnt


@pytest.mark.parametrize("R,E,k", [(2, 8, 2), (4, 20, 4), (8, 20, 4), (3, 7, 2)])
def test_plan_layout_is_consistent_across_ranks(R, E, k):
    T = 300
    cnt = _random_counts(R, E, T, k, seed=R * 100 + E)
    cap = receive_capacity(T, k, E, R)
    plans = [plan_reference(cnt, r, cap) for r in range(R)]
    for d in range(R):
        lo, hi = expert_range(d, E, R)
        _, row_off, recv_cnt, tile_group = plans[d]
        # per local expert: a 128-aligned range large enough for all sources' rows
        for l in range(hi - lo):
            assert int(row_off[l]) % 256 == 0
            assert int(row_off[l + 1]) - int(row_off[l]) == (int(recv_cnt[l]) + 255) // 256 * 256
            assert int(recv_cnt[l]) == int(cnt[:, lo + l].sum())
        # the rows every source writes for expert e are disjoint and inside e's range
        for e in range(lo, hi):
            l = e - lo
            spans = sorted((int(plans[s][0][e]), int(plans[s][0][e]) + int(cnt[s, e])) for s in range(R))
            assert spans[0][0] == int(row_off[l])
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            assert spans[-1][1] == int(row_off[l]) + int(recv_cnt[l])
        # tiles map to the expert whose range holds them; unused tiles are -1
        used = int(row_off[-1])
        for i, g in enumerate(tile_group.tolist()):
            row = i * 128
            if row >= used:
                assert g == -1
            else:
                assert int(row_off[g]) <= row < int(row_off[g + 1])


def test_plan_skips_empty_experts():
    cnt = torch.tensor([[5, 0, 0, 3], [0, 0, 2, 1]], dtype=torch.int32)
    cap = receive_capacity(8, 2, 4, 2)
    send_base, row_off, recv_cnt, tg = plan_reference(cnt, 0, cap)
    assert row_off.tolist() == [0, 256, 256]
    assert recv_cnt.tolist() == [5, 0]
    assert (tg[:2] == 0).all() and (tg[2:] == -1).all()   # one 256-row range = two 128-row tiles
    # rank 1 receives experts 2, 3; rank 1's rows for expert 3 follow rank 0's 3 rows
    _, row_off1, _, _ = plan_reference(cnt, 1, cap)
    sb1, _, _, _ = plan_reference(cnt, 1, cap)
    assert row_off1.tolist() == [0, 256, 512]
    assert sb1[3] == 256 + 3 and send_base[3] == 256


@pytest.mark.parametrize("R,E,k", [(2, 8, 2), (8, 20, 4), (8, 64, 6), (3, 5, 3), (8, 8, 1)])
def test_balanced_plan_covers_every_row_once(R, E, k):
    from parallel.ep import balanced_capacity, plan_reference_balanced
    T = 333
    g = torch.Generator().manual_seed(R * 100 + E)
    # skewed routing: a few experts take most rows (as at random init)
    logits = torch.randn(R, T, E, generator=g) + torch.linspace(0, 3, E)
    idx = logits.topk(k, dim=-1).indices
    cnt = torch.stack([torch.bincount(idx[s].flatten(), minlength=E) for s in range(R)]).to(torch.int32)
    cap = balanced_capacity(T, k, E, R)
    plans = [plan_reference_balanced(cnt, r) for r in range(R)]
    chunk = plans[0][3]
    assert all(p[3] == chunk for p in plans) and chunk % 256 == 0 and chunk <= cap
    tot = cnt.sum(0)
    # every rank computes at most one share; shares differ only at the tail
    used = [p[4] for p in plans]
    assert sum(used) == int(((tot + 255) // 256 * 256).sum())
    assert max(used) <= chunk
    # simulate the dispatch: every (source, expert) row lands in a real-row slot of its expert
    seen = {d: set() for d in range(R)}
    for s in range(R):
        send_base = plans[s][0]
        for e in range(E):
            for j in range(int(cnt[s, e])):
                gp = int(send_base[e]) + j
                d, row = gp // chunk, gp % chunk
                _, row_off, recv_cnt, _, _ = plans[d]
                assert int(row_off[e]) <= row < int(row_off[e]) + int(recv_cnt[e])
                assert row not in seen[d]
                seen[d].add(row)
    for d in range(R):
        _, row_off, recv_cnt, _, u = plans[d]
        assert len(seen[d]) == int(recv_cnt.sum())
        assert torch.all(row_off[1:] >= row_off[:-1]) and int(row_off[-1]) == u
        # 256-row alignment of every expert boundary inside a share (CTA-pair tiles stay in one expert)
        assert all(int(v) % 256 == 0 for v in row_off)
