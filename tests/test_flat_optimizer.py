"""Host logic of the flat AdamW optimizer on CPU: sharded (ZeRO-1) moments and
the learning-rate schedule when the data-parallel step replaces the local
update.  The kernel library is replaced by a fake of its one host-visible call
here (``cast_f32_bf16``); no kernel runs."""
import copy
import warnings

import pytest
import torch
import torch.nn as nn
from torch.optim.lr_scheduler import LambdaLR

import ops.flat as flat
from training.pretrain import make_warmup_cosine_lambda


class _FakeNative:
    @staticmethod
    def cast_f32_bf16(src, dst):
        dst.copy_(src)


@pytest.fixture
def cpu_flat(monkeypatch):
    monkeypatch.setattr(flat, "native", lambda: _FakeNative())
    torch.manual_seed(0)
    params = [nn.Parameter(torch.randn(10, 7)), nn.Parameter(torch.randn(33)), nn.Parameter(torch.randn(5, 40))]
    fp = flat.FlatParams([[params[0]], [params[1], params[2]]], "cpu")
    return params, fp


def _opt(params, fp):
    return flat.FlatAdamW([{"params": params, "weight_decay": 0.1}], [fp], lr=1e-3)


def test_sharded_moments_load_and_gather(cpu_flat):
    params, fp = cpu_flat
    full = _opt(params, fp)
    full.exp_avg[0].copy_(torch.arange(fp.numel, dtype=torch.float32))
    full.exp_avg_sq[0].copy_(torch.arange(fp.numel, dtype=torch.float32) * 0.5)
    full.step_count = 4
    full._bind_state()
    sd = copy.deepcopy(full.state_dict())
    cuts = [(0, 64), (64, 192), (192, fp.numel)]
    pieces_m, pieces_v = [], []
    for lo, hi in cuts:
        opt = _opt(params, fp)
        opt.shard_moments(0, lo, hi)
        assert opt.exp_avg[0].numel() == hi - lo
        assert all("exp_avg" not in st for st in opt.state.values())   # nothing full-size is bound
        opt.load_state_dict(sd)
        assert opt.step_count == 4
        pieces_m.append(opt.exp_avg[0])
        pieces_v.append(opt.exp_avg_sq[0])
    gathered = (torch.cat(pieces_m), torch.cat(pieces_v))
    # padding between blocks is not part of any parameter: compare parameter elements only
    for p in params:
        o = fp.offsets[id(p)]
        assert torch.equal(gathered[0][o:o + p.numel()], full.exp_avg[0][o:o + p.numel()])
        assert torch.equal(gathered[1][o:o + p.numel()], full.exp_avg_sq[0][o:o + p.numel()])
    # binding the gathered buffers reproduces the unsharded checkpoint layout
    opt.step_count = 4
    opt._bind_state({0: gathered})
    again = opt.state_dict()
    for i, st in sd["state"].items():
        assert torch.equal(again["state"][i]["exp_avg"], st["exp_avg"])
        assert torch.equal(again["state"][i]["exp_avg_sq"], st["exp_avg_sq"])


def test_stepper_gets_the_single_process_lr_schedule(cpu_flat):
    params, fp = cpu_flat
    opt = _opt(params, fp)
    lam = make_warmup_cosine_lambda(3, 12, 0.05)
    applied = []
    opt.stepper = lambda o: applied.append(o.param_groups[0]["lr"])
    sched = LambdaLR(opt, lam)
    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        for _ in range(8):
            opt.step()
            sched.step()
    assert applied == pytest.approx([1e-3 * lam(k) for k in range(8)], rel=0, abs=1e-15)
    assert not any("lr_scheduler.step()" in str(w.message) for w in caught)
