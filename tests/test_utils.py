"""CPU tests of the checkpoint manager and memory estimator."""
import os
from unittest.mock import patch

import pytest
import torch

from models.transformer import Transformer
from utils.checkpoint import CheckpointManager
from utils import memory


def _opt(m):
    return torch.optim.AdamW(m.parameters(), lr=1e-3)


class TestCheckpointManager:
    def test_save_load_and_latest(self, small_cfg, tmp_dir):
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        mgr.save(m, _opt(m), 3, extra_meta={"step": 99, "x": 1})
        mgr.save(m, _opt(m), 5)
        assert mgr.latest_step() == 5
        m2 = Transformer(small_cfg)
        meta = mgr.load(m2, 3, device="cpu", optimizer=_opt(m2), strict=False)
        assert meta == {"step": 3, "x": 1}
        for a, b in zip(m.state_dict().values(), m2.state_dict().values()):
            assert torch.equal(a, b)

    def test_incomplete_ignored(self, small_cfg, tmp_dir):
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        mgr.save(m, _opt(m), 2)
        mgr.save(m, _opt(m), 4)
        os.remove(tmp_dir / "optim_step_4.pt")
        assert mgr.latest_step() == 2

    def test_missing_raises(self, small_cfg, tmp_dir):
        with pytest.raises(FileNotFoundError):
            CheckpointManager(str(tmp_dir)).load(Transformer(small_cfg), 1, device="cpu")

    def test_tied_saved_once(self, small_cfg, tmp_dir):
        from safetensors.torch import load_file
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        mgr.save(m, _opt(m), 1)
        keys = load_file(str(tmp_dir / "model_step_1.safetensors")).keys()
        assert ("embed.weight" in keys) != ("head.weight" in keys)
        m2 = Transformer(small_cfg)
        mgr.load(m2, 1, device="cpu", strict=False)
        assert m2.head.weight.data_ptr() == m2.embed.weight.data_ptr()
        assert torch.equal(m2.head.weight, m.head.weight)

    def test_expert_shards_merge_and_completeness(self, small_cfg, tmp_dir):
        """A step saved with routed experts sharded over two ranks: the model
        file without them, one shard file per rank; the step is complete only
        with every shard, and an unsharded load merges the shards' weights."""
        m = Transformer(small_cfg)
        full = m.state_dict()
        experts = {k: v for k, v in full.items() if ".experts." in k}
        assert experts, "the test config needs routed experts"
        mgr = CheckpointManager(str(tmp_dir))
        E = small_cfg["n_routed_experts"]
        for r in range(2):
            lo, hi = r * E // 2, (r + 1) * E // 2
            mine = {k: v for k, v in experts.items() if lo <= int(k.split(".experts.")[1].split(".")[0]) < hi}
            shard = dict(mine)
            shard.update({"exp_avg." + k: torch.zeros_like(v) for k, v in mine.items()})
            shard.update({"exp_avg_sq." + k: torch.ones_like(v) for k, v in mine.items()})
            mgr.save_expert_shard(7, r, 2, shard)
        mgr.save(m, _opt(m), 7, extra_meta={"expert_shards": 2},
                 state_dict={k: v for k, v in full.items() if k not in experts})
        assert mgr.latest_step() == 7
        m2 = Transformer(small_cfg)
        mgr.load(m2, 7, device="cpu", strict=False)   # tied head.weight is written once
        for k, v in m2.state_dict().items():
            assert torch.equal(v, full[k]), k
        back = mgr.load_expert_shard(7, 1, 2)
        assert all(torch.equal(back["exp_avg_sq." + k], torch.ones_like(experts[k]))
                   for k in back if not k.startswith("exp_avg"))
        os.remove(mgr.expert_shard_path(7, 1, 2))
        assert mgr.latest_step() is None

    def test_crash_leaves_no_temp(self, small_cfg, tmp_dir):
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        with patch("utils.checkpoint.save_file", side_effect=OSError("disk full")):
            with pytest.raises(OSError):
                mgr.save(m, _opt(m), 1)
        assert list(tmp_dir.iterdir()) == []
        assert mgr.latest_step() is None

    def test_strict(self, small_cfg, tmp_dir):
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        state = dict(m.state_dict())
        state["bogus"] = torch.zeros(1)
        mgr.save(m, _opt(m), 1, state_dict=state)
        with pytest.raises(RuntimeError, match="missing|unexpected"):
            mgr.load(Transformer(small_cfg), 1, device="cpu", strict=True)
        mgr.load(Transformer(small_cfg), 1, device="cpu", strict=False)
        untied = {**small_cfg, "weight_tying": False}
        mu = Transformer(untied)
        mgr.save(mu, _opt(mu), 2)
        mgr.load(Transformer(untied), 2, device="cpu", strict=True)


class TestMemory:
    def test_components(self, small_cfg):
        m = Transformer(small_cfg)
        n = sum(p.numel() for p in set(m.parameters()))
        assert memory._parameter_bytes(m) == 2 * n and memory._optimiser_bytes(m) == 12 * n
        assert memory._kv_cache_bytes(m, 10, 2) == 2 * 10 * (16 + 4) * 2 * small_cfg["n_layers"]
        assert memory._activation_bytes(10, 2, 64, 2, True) == 24 * 10 * 2 * 64 * 2 * 2
        assert memory._activation_bytes(10, 2, 64, 2, False) == 36 * 10 * 2 * 64 * 2 * 2
        assert memory._infer_dim_n_layers(m) == (64, 2)
        assert memory._infer_dim_n_layers(torch.nn.Linear(2, 2)) == (0, 0)

    def test_estimates(self, small_cfg):
        m = Transformer(small_cfg)
        a = memory.estimate_model_memory_gb(m, 64, 1, overhead_gb=0.0)
        b = memory.estimate_model_memory_gb(m, 64, 8, overhead_gb=0.0)
        inf = memory.estimate_model_memory_gb(m, 64, 8, overhead_gb=0.0, inference=True)
        assert 0 < a < b and inf < b
        assert memory._detect_overhead_gb() == 2.0

    def test_fit_assertion(self, monkeypatch):
        memory.assert_fits_in_available_gpu(1e9)  # no CUDA: no-op
        class Props:
            total_memory = 8 * 1024 ** 3
        monkeypatch.setattr(memory.torch.cuda, "is_available", lambda: True)
        monkeypatch.setattr(memory.torch.cuda, "get_device_properties", lambda i: Props())
        with pytest.raises(RuntimeError):
            memory.assert_fits_in_available_gpu(7.5, safety_margin_gb=1.0)
        memory.assert_fits_in_available_gpu(6.0, safety_margin_gb=1.0)

    def test_sharded_estimate_shrinks(self, small_cfg):
        m = Transformer(small_cfg)
        assert memory.estimate_sharded_training_gb(m, 64, 2, 4, 4) < memory.estimate_sharded_training_gb(m, 64, 2)


def test_consolidate_sharded_experts(small_cfg, tmp_dir):
    """A checkpoint saved with routed experts sharded over two ranks (model
    and optimizer files without experts, one shard file per rank) merges back
    into the plain checkpoint an unsharded trainer writes: same weights, same
    optimizer state at the single-process parameter indices."""
    from dataclasses import asdict
    from models.mtp import MultiTokenPrediction
    from training.consolidate import consolidate, optimizer_index
    from training.pretrain import TrainingConfig, _unique_params
    from safetensors.torch import load_file

    torch.manual_seed(0)
    raw = Transformer(small_cfg)
    wrap = MultiTokenPrediction(small_cfg, raw)
    params = _unique_params(wrap)
    opt = torch.optim.AdamW([{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
                             {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}], lr=1e-3)
    for p in params:
        p.grad = torch.randn_like(p)
    opt.step()
    full = {k: v for k, v in raw.state_dict().items() if k != "head.weight"}
    full.update({"mtp." + k: v for k, v in wrap.state_dict().items() if k.startswith("mtp_modules.")})
    full_opt = opt.state_dict()
    index = optimizer_index(small_cfg, has_mtp=True)
    assert sorted(index.values()) == list(range(len(params)))

    # what the sharded trainer writes (two ranks, two experts each)
    mgr = CheckpointManager(str(tmp_dir / "sharded"))
    E = small_cfg["n_routed_experts"]
    experts = [k for k in full if ".experts." in k]
    for r in range(2):
        lo, hi = r * E // 2, (r + 1) * E // 2
        shard = {}
        for k in experts:
            if lo <= int(k.split(".experts.")[1].split(".")[0]) < hi:
                st = full_opt["state"][index[k]]
                shard.update({k: full[k], "exp_avg." + k: st["exp_avg"], "exp_avg_sq." + k: st["exp_avg_sq"]})
        mgr.save_expert_shard(4, r, 2, shard)
    opt_sharded = {"state": {i: v for i, v in full_opt["state"].items() if i not in {index[k] for k in experts}},
                   "param_groups": full_opt["param_groups"]}
    meta = {"expert_shards": 2, "has_mtp": True, "config": asdict(TrainingConfig(model_config=dict(small_cfg)))}
    mgr.save(raw, opt, 4, extra_meta=meta, state_dict={k: v for k, v in full.items() if k not in experts},
             optimizer_state=opt_sharded)

    assert consolidate(str(tmp_dir / "sharded"), str(tmp_dir / "plain")) == 4
    plain = CheckpointManager(str(tmp_dir / "plain"))
    assert plain.latest_step() == 4
    w = load_file(str(tmp_dir / "plain" / "model_step_4.safetensors"))
    written = CheckpointManager._unique_storage(full)   # tied tensors are written once
    assert w.keys() == written.keys() and all(torch.equal(w[k], written[k]) for k in written)
    got = torch.load(tmp_dir / "plain" / "optim_step_4.pt", weights_only=True)
    assert got["state"].keys() == full_opt["state"].keys()
    for i, st in full_opt["state"].items():
        for name in ("exp_avg", "exp_avg_sq", "step"):
            assert torch.equal(got["state"][i][name], st[name]), (i, name)
    # a fresh single-process model and optimizer load it
    raw2 = Transformer(small_cfg)
    wrap2 = MultiTokenPrediction(small_cfg, raw2)
    p2 = _unique_params(wrap2)
    opt2 = torch.optim.AdamW([{"params": [p for p in p2 if p.dim() >= 2], "weight_decay": 0.1},
                              {"params": [p for p in p2 if p.dim() < 2], "weight_decay": 0.0}], lr=1e-3)
    plain.load(raw2, 4, device="cpu", optimizer=opt2, strict=False)
    assert torch.equal(raw2.layers[1].ffn.experts[3].w2.weight, raw.layers[1].ffn.experts[3].w2.weight)
    with pytest.raises(ValueError):
        consolidate(str(tmp_dir / "plain"), str(tmp_dir / "again"))


def test_scaled_config_fits_only_with_sharded_experts():
    """The 14B scaled config (instantiated on the meta device): ~12.7B routed
    expert parameters; one B200 (180 GB) cannot hold it with AdamW state when
    experts are replicated, eight ranks with sharded experts can."""
    import yaml
    from pathlib import Path
    cfg = yaml.safe_load(open(Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200" / "configs"
                              / "scaled_13b.yaml"))
    with torch.device("meta"):
        m = Transformer(cfg["model"])
    experts = sum(p.numel() for n, p in m.named_parameters() if ".experts." in n)
    total = sum(p.numel() for p in m.parameters())
    assert 12.5e9 < experts < 13.0e9 and 13.5e9 < total < 14.2e9
    S, B = cfg["model"]["max_seq_len"], cfg["training"]["micro_batch_size"]
    assert memory.estimate_sharded_training_gb(m, S, B, ep_size=1, dp_size=8) > 180
    assert memory.estimate_sharded_training_gb(m, S, B, ep_size=8, dp_size=8) < 120


def test_expert_sharding_hint():
    """The start-up hint names expert sharding exactly when it would make the
    scaled config fit a 180 GB device on 8 ranks."""
    import yaml
    from pathlib import Path
    cfg = yaml.safe_load(open(Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200" / "configs"
                              / "scaled_13b.yaml"))
    with torch.device("meta"):
        m = Transformer(cfg["model"])
    S, B = cfg["model"]["max_seq_len"], cfg["training"]["micro_batch_size"]
    hint = memory.expert_sharding_hint(m, S, B, world_size=8, ep_size=0, shard_experts=False, device_gb=180)
    assert hint is not None and "shard_experts: true" in hint
    assert memory.expert_sharding_hint(m, S, B, world_size=8, ep_size=0, shard_experts=True, device_gb=180) is None
    one = memory.expert_sharding_hint(m, S, B, world_size=1, ep_size=1, shard_experts=False, device_gb=180)
    assert one is not None and "shard_experts" not in one


class TestBackgroundCheckpoint:
    def test_background_save_round_trip_and_visibility(self, small_cfg, tmp_dir):
        """A background save snapshots the step, reports it complete only once
        every file is written, and loads like a synchronous one."""
        import threading
        from safetensors.torch import save_file as real_save_file
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        gate = threading.Event()

        def slow_save_file(tensors, path):
            gate.wait(10)
            real_save_file(tensors, path)

        want = {k: v.clone() for k, v in m.state_dict().items()}
        with patch("utils.checkpoint.save_file", side_effect=slow_save_file):
            mgr.save(m, _opt(m), 6, background=True)
            with torch.no_grad():
                for p in m.parameters():
                    p.add_(1.0)          # training goes on: the snapshot must not see this
            assert mgr.latest_step() is None
            gate.set()
            mgr.wait()
        assert mgr.latest_step() == 6
        m2 = Transformer(small_cfg)
        mgr.load(m2, 6, device="cpu", strict=False)
        for k, v in m2.state_dict().items():
            assert torch.equal(v, want[k]), k

    def test_background_error_surfaces_on_wait(self, small_cfg, tmp_dir):
        m = Transformer(small_cfg)
        mgr = CheckpointManager(str(tmp_dir))
        with patch("utils.checkpoint.save_file", side_effect=OSError("disk full")):
            mgr.save(m, _opt(m), 1, background=True)
            with pytest.raises(RuntimeError, match="background checkpoint write failed"):
                mgr.wait()
        assert list(tmp_dir.iterdir()) == [] and mgr.latest_step() is None
        mgr.wait()   # the error is reported once
