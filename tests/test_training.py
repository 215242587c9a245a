"""CPU tests of the trainer, dataset, schedule, checkpoint round trips and NaN guard."""
import json
from dataclasses import asdict
from unittest.mock import patch

import pytest
import torch
import yaml

from models.transformer import count_parameters
from training.pretrain import (Pretrainer, PretrainDataset, TrainingConfig, config_from_yaml,
                               make_warmup_cosine_lambda)


def _cfg(small_cfg, ckpt, **kw):
    base = dict(model_config=small_cfg, data_path="/nonexistent", checkpoint_dir=str(ckpt),
                max_seq_len=small_cfg["max_seq_len"], vocab_size=small_cfg["vocab_size"], batch_size=2,
                gradient_accumulation_steps=2, max_steps=4, warmup_steps=1, lr=1e-3, weight_decay=0.0,
                grad_checkpoint=False, compile_model=False, nan_guard=False, save_every=10, log_every=10)
    base.update(kw)
    return TrainingConfig(**base)


def test_config_defaults_and_serialisable():
    c = TrainingConfig()
    assert (c.lr, c.weight_decay, c.beta1, c.beta2, c.max_grad_norm) == (2.2e-4, 0.1, 0.9, 0.95, 1.0)
    assert c.bias_update_every == 10 and c.mtp_weight == 0.0 and c.seed == 42
    json.dumps(asdict(c))


def test_schedule_points():
    f = make_warmup_cosine_lambda(10, 110, 0.1)
    assert f(0) == 0.0 and f(5) == 0.5 and f(10) == 1.0
    assert abs(f(60) - (0.1 + 0.9 * 0.5)) < 1e-9
    assert f(110) == 0.1 and f(500) == 0.1
    assert make_warmup_cosine_lambda(0, 10, 0.2)(0) == 1.0


class TestDataset:
    def test_single_file_windows(self, token_file):
        ds = PretrainDataset(token_file, 32, 1024)
        assert len(ds) == (512 - 1) // 32
        x, y = ds[3]
        assert x.shape == (32,) and torch.equal(x[1:], y[:-1])

    def test_shards_cross_boundaries(self, shard_dir):
        ds = PretrainDataset(shard_dir, 50, 1024)
        assert len(ds) == (384 - 1) // 50
        x, y = ds[2]   # tokens 100..150 span shard 0 and 1
        assert torch.equal(x, torch.arange(100, 150)) and torch.equal(y, torch.arange(101, 151))

    def test_locate(self, shard_dir):
        ds = PretrainDataset(shard_dir, 50, 1024)
        assert ds._locate(0) == (0, 0) and ds._locate(128) == (1, 0) and ds._locate(383) == (2, 127)
        for bad in (-1, 384):
            with pytest.raises(IndexError):
                ds._locate(bad)

    def test_missing(self):
        with pytest.raises(FileNotFoundError):
            PretrainDataset("/no/such/file.bin", 8, 10)


class TestPretrainer:
    def test_construct_and_groups(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir))
        assert tr.mtp_wrapper is None and tr.device.type == "cpu"
        n_opt = sum(p.numel() for g in tr.optimizer.param_groups for p in g["params"])
        assert n_opt == sum(p.numel() for p in set(tr.model.parameters()))
        assert all(p.dim() >= 2 for p in tr.optimizer.param_groups[0]["params"])
        assert all(p.dim() < 2 for p in tr.optimizer.param_groups[1]["params"])

    def test_mtp_enabled_only_with_weight(self, small_cfg, tmp_dir):
        assert Pretrainer(_cfg(small_cfg, tmp_dir, mtp_weight=0.3)).mtp_wrapper is not None

    def test_mup(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir, mup_lr=True))
        total, _ = count_parameters(tr.raw_model)
        assert abs(tr.config.lr - 6e-4 * (757226496 / total) ** 0.5) < 1e-12

    def test_scheduler_horizon(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir, max_steps=8, warmup_steps=0, min_lr_ratio=0.1))
        t = torch.randint(0, small_cfg["vocab_size"], (2, small_cfg["max_seq_len"]))
        for i in range(8):
            tr.train_step(t, t, i)
        assert tr._opt_steps == 4
        assert abs(tr.scheduler.get_last_lr()[0] - 1e-3 * 0.1) < 1e-12

    def test_step_updates_and_bias(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir, gradient_accumulation_steps=1, bias_update_every=1, warmup_steps=0,
                             mtp_weight=0.3))
        before = {n: p.detach().clone() for n, p in tr.raw_model.named_parameters()}
        bias0 = [m.gate.bias.clone() for m in tr.raw_model.moe_layers()]
        t = torch.randint(0, small_cfg["vocab_size"], (2, 32))
        out = tr.train_step(t, t, 0)
        assert torch.isfinite(out["loss"]) and out["mtp_loss"] is not None
        changed = [n for n, p in tr.raw_model.named_parameters() if not torch.equal(p, before[n])]
        assert "layers.0.attn.wkv_a.weight" in changed
        assert any(not torch.equal(b, m.gate.bias) for b, m in zip(bias0, tr.raw_model.moe_layers()))

    def test_nan_guard(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir, nan_guard=True, gradient_accumulation_steps=1))
        t = torch.randint(0, small_cfg["vocab_size"], (1, 4))
        bad = lambda *a, **k: torch.full((1, 4, small_cfg["vocab_size"]), float("nan"))
        with patch.object(tr.model, "forward", side_effect=bad):
            assert tr.train_step(t, t, 0) is None

    def test_nan_streak_rolls_back(self, small_cfg, tmp_dir, token_file):
        cfg = _cfg(small_cfg, tmp_dir, nan_guard=True, nan_guard_max_consecutive=2, gradient_accumulation_steps=1,
                   data_path=token_file, max_seq_len=16, max_steps=3)
        tr = Pretrainer(cfg)
        tr.save_checkpoint(1)
        calls = []
        real = tr.load_checkpoint
        bad = lambda *a, **k: torch.full((2, 16, small_cfg["vocab_size"]), float("nan"))

        def spy(step):
            calls.append(step)
            tr.model.forward = tr.model.__class__.forward.__get__(tr.model)
            return real(step)

        with patch.object(tr, "load_checkpoint", side_effect=spy):
            tr.model.forward = bad
            tr.train()
        assert calls and calls[0] == 1

    def test_nan_without_checkpoint_raises(self, small_cfg, tmp_dir, token_file):
        cfg = _cfg(small_cfg, tmp_dir, nan_guard=True, nan_guard_max_consecutive=1, gradient_accumulation_steps=1,
                   data_path=token_file, max_seq_len=16, max_steps=3)
        tr = Pretrainer(cfg)
        tr.model.forward = lambda *a, **k: torch.full((2, 16, small_cfg["vocab_size"]), float("nan"))
        with pytest.raises(RuntimeError, match="no checkpoint"):
            tr.train()


def test_corrupted_latest_checkpoint_does_not_stop_training(small_cfg, tmp_dir, token_file):
    """A latest checkpoint whose weight file is corrupted (a crash outside the
    atomic write, a bad disk) is reported and training starts fresh, as the
    reference's loop does; the run still reaches max_steps and saves."""
    cfg = _cfg(small_cfg, tmp_dir, gradient_accumulation_steps=1, data_path=token_file, max_seq_len=16, max_steps=3)
    tr = Pretrainer(cfg)
    tr.save_checkpoint(2)
    wpath = tmp_dir / "model_step_2.safetensors"
    wpath.write_bytes(wpath.read_bytes()[:64])          # truncated: unreadable
    tr2 = Pretrainer(cfg)
    logged = []
    real_log = tr2._log
    tr2._log = lambda msg: (logged.append(msg), real_log(msg))
    tr2.train()
    assert any("Could not load checkpoint" in m for m in logged)
    assert tr2.ckpt_manager.latest_step() == 3


class TestCheckpointRoundTrip:
    def test_weights_optimizer_meta(self, small_cfg, tmp_dir):
        tr = Pretrainer(_cfg(small_cfg, tmp_dir, mtp_weight=0.3, gradient_accumulation_steps=1))
        t = torch.randint(0, small_cfg["vocab_size"], (2, 32))
        tr.train_step(t, t, 0)
        tr.save_checkpoint(7)
        meta = json.load(open(tmp_dir / "meta_step_7.json"))
        assert meta["step"] == 7 and meta["opt_steps"] == 1 and meta["has_mtp"] is True
        from safetensors.torch import load_file
        keys = load_file(str(tmp_dir / "model_step_7.safetensors")).keys()
        assert "head.weight" not in keys and any(k.startswith("mtp.mtp_modules.0.block.") for k in keys)
        assert all(v.dtype == torch.float32 for v in load_file(str(tmp_dir / "model_step_7.safetensors")).values())
        tr2 = Pretrainer(_cfg(small_cfg, tmp_dir, mtp_weight=0.3, gradient_accumulation_steps=1))
        assert tr2.load_checkpoint(7) == 7 and tr2._opt_steps == 1
        for (n, a), (_, b) in zip(tr.mtp_wrapper.named_parameters(), tr2.mtp_wrapper.named_parameters()):
            assert torch.equal(a, b), n
        assert tr2.raw_model.head.weight.data_ptr() == tr2.raw_model.embed.weight.data_ptr()


def test_yaml_mapping(small_cfg, tmp_dir):
    y = {"model": small_cfg, "training": {"micro_batch_size": 3, "total_steps": 9, "grad_clip": 0.5,
                                          "mtp_loss_weight": 0.3, "log_interval": 7, "save_interval": 11},
         "data": {"train_data_path": "/d"}}
    c = config_from_yaml(y)
    assert (c.batch_size, c.max_steps, c.max_grad_norm, c.mtp_weight, c.log_every, c.save_every) == (3, 9, 0.5, 0.3, 7, 11)
    assert c.data_path == "/d" and c.max_seq_len == small_cfg["max_seq_len"]
    assert config_from_yaml(y, no_checkpoint=True).grad_checkpoint is False


def test_step_diagnostics_report_expert_load(small_cfg, tmp_dir):
    tr = Pretrainer(_cfg(small_cfg, tmp_dir / "ck"))
    tok = torch.randint(0, small_cfg["vocab_size"], (2, 33))
    tr.train_step(tok[:, :-1], tok[:, 1:], 0)
    hist = tr.expert_load_histograms()
    assert hist and all(len(c) == small_cfg["n_routed_experts"] for c in hist.values())
    assert all(sum(c) == 2 * 32 * small_cfg["n_activated_experts"] for c in hist.values())
    d = tr.step_diagnostics()
    assert d["expert_load_max_over_mean"] >= 1.0


def test_small_shard_builder_feeds_pretrain_dataset(tmp_path):
    """Synthetic source + byte tokenizer -> shard_0000.bin (uint32), read by
    PretrainDataset; the synthetic source is identical run to run."""
    from data.build_small_shard import build_shard, open_source, open_tokenizer, synthetic_documents
    from training.pretrain import PretrainDataset
    encode, eos, vocab = open_tokenizer("bytes")
    path = build_shard(str(tmp_path), open_source("synthetic"), encode, eos, target_tokens=5000)
    t = torch.load(path, weights_only=True)
    assert t.dtype == torch.uint32 and t.numel() == 5000 and int(t.long().max()) <= eos
    assert list(synthetic_documents(3)) == list(synthetic_documents(3))
    ds = PretrainDataset(str(tmp_path), max_seq_len=64, vocab_size=vocab)
    x, y = ds[3]
    x, y = x.long(), y.long()
    assert len(ds) == (5000 - 1) // 64 and x.shape == (64,) and torch.equal(x[1:], y[:-1])


def test_prepare_data_without_external_pipeline(tmp_path):
    import yaml
    from data import prepare_data
    out = tmp_path / "data_config.yaml"
    rc = prepare_data.main(["--config-out", str(out)])
    cfg = yaml.safe_load(out.read_text())
    assert rc == 2 and cfg["pipeline"]["tokenizer"]["vocab_size"] == 100_018
    assert cfg["pipeline"]["tokenizer"]["eos_token_id"] == 100_017


def test_scaled_config_parallel_section():
    """The scaled config's `parallel:` section reaches the trainer: experts over
    all ranks, sharded, receive buffers at twice the mean load."""
    import yaml
    from pathlib import Path
    y = yaml.safe_load(open(Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200" / "configs"
                            / "scaled_13b.yaml"))
    c = config_from_yaml(y)
    assert c.ep_size == 0 and c.ep_shard_experts is True and c.ep_capacity_factor == 2.0
    c412 = config_from_yaml(yaml.safe_load(open(Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200"
                                                / "configs" / "pretrain_412m.yaml")))
    assert c412.ep_shard_experts is False


def test_async_checkpoint_training_loop(small_cfg, tmp_dir, token_file):
    """With async_checkpoint the loop's periodic and final checkpoints are
    written by the background writer and complete when train() returns."""
    cfg = _cfg(small_cfg, tmp_dir, gradient_accumulation_steps=1, data_path=token_file, max_seq_len=16, max_steps=4,
               save_every=2, async_checkpoint=True)
    tr = Pretrainer(cfg)
    tr.train()
    assert tr.ckpt_manager.latest_step() == 4 and 2 in tr.ckpt_manager._list_steps()
    tr2 = Pretrainer(cfg)
    assert tr2.load_checkpoint(4) == 4
    for (n, a), (_, b) in zip(tr.raw_model.named_parameters(), tr2.raw_model.named_parameters()):
        assert torch.equal(a, b), n


def test_tiny_benchmark_script_runs_on_cpu():
    """training/bench_tiny.py (the tiny-config step + decode benchmark) prints
    its JSON line; on the CPU it runs this package's PyTorch path."""
    import subprocess
    import sys as _sys
    from pathlib import Path
    pkg = Path(__file__).resolve().parent.parent / "deepseek-v3-lite_b200"
    r = subprocess.run([_sys.executable, "training/bench_tiny.py", "--steps", "1", "--new", "2"], cwd=pkg,
                       capture_output=True, text=True, timeout=600, env={**__import__("os").environ,
                                                                         "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "ours" and line["step_ms"] > 0 and line["decode_tokens"] == 2
