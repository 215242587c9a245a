"""CPU tests of speculative decoding, per-row decode and the CLI helpers."""
import pytest
import torch
import yaml

from inference.generate import load_config, resolve_checkpoint
from inference.speculative import BatchedSpeculativeDecoder, SpeculativeDecoder
from models.mtp import MultiTokenPrediction
from models.transformer import Transformer
from ops.decode import batched_decode_step
from utils.checkpoint import CheckpointManager


@pytest.fixture()
def models(small_cfg):
    torch.manual_seed(0)
    m = Transformer(small_cfg).eval()
    mt = MultiTokenPrediction(small_cfg, m)
    return m, mt.mtp_modules[0]


def test_generate_step_and_cache(models, small_cfg):
    m, mtp = models
    sd = SpeculativeDecoder(m, mtp, 0.8)
    p = torch.randint(0, small_cfg["vocab_size"], (1, 6))
    m.reset_cache()
    m(p, start_pos=0, use_cache=True)
    tm, td, ok = sd.generate_step(p[:, -1:], start_pos=5, temperature=0.0)
    assert tm.shape == (1,) and td.shape == (1,) and isinstance(ok, bool)
    assert m.layers[0].attn.kv_cache[0, 6].abs().sum() > 0


def test_threshold_extremes(models, small_cfg):
    m, mtp = models
    p = torch.randint(0, small_cfg["vocab_size"], (1, 4))
    always = SpeculativeDecoder(m, mtp, 0.0).generate(p, 8, temperature=0)
    never = SpeculativeDecoder(m, mtp, 1e9).generate(p, 8, temperature=0)
    assert always.shape[1] == never.shape[1] == 12
    # With a never-accept threshold every token comes from the main model: plain greedy.
    assert torch.equal(never, m.generate(p, 8, temperature=0))


def test_eos_stops(models, small_cfg):
    m, mtp = models
    p = torch.randint(0, small_cfg["vocab_size"], (1, 4))
    first = m.generate(p, 1, temperature=0)[0, -1].item()
    out = SpeculativeDecoder(m, mtp, 1e9).generate(p, 8, temperature=0, eos_token_id=first)
    assert out.shape[1] == 5


def test_batched_matches_single(models, small_cfg):
    m, mtp = models
    prompts = torch.randint(0, small_cfg["vocab_size"], (3, 5))
    buf, lens = BatchedSpeculativeDecoder(m, mtp, 0.8).generate(prompts, max_new_tokens=6)
    for b in range(3):
        single = SpeculativeDecoder(m, mtp, 0.8).generate(prompts[b:b + 1], 6, temperature=0)
        n = int(lens[b])
        assert n == 11 and torch.equal(buf[b, :n], single[0, :n])


def test_row_decode_matches_forward(models, small_cfg):
    m, _ = models
    t = torch.randint(0, small_cfg["vocab_size"], (2, 9))
    full = m(t, use_cache=False)
    m.reset_cache()
    m(t[:, :8], start_pos=0, use_cache=True)
    logits, _ = batched_decode_step(m, t[:, 8], torch.tensor([8, 8]))
    assert torch.allclose(logits, full[:, 8], atol=1e-5)


def test_load_config(tmp_dir, small_cfg):
    good = tmp_dir / "c.yaml"
    good.write_text(yaml.safe_dump({"model": small_cfg}))
    assert load_config(str(good))["model"]["dim"] == small_cfg["dim"]
    bad = tmp_dir / "b.yaml"
    bad.write_text(yaml.safe_dump({"training": {}}))
    with pytest.raises(ValueError):
        load_config(str(bad))
    with pytest.raises(FileNotFoundError):
        load_config(str(tmp_dir / "none.yaml"))


def test_resolve_checkpoint(tmp_dir, small_cfg):
    m = Transformer(small_cfg)
    mgr = CheckpointManager(str(tmp_dir))
    mgr.save(m, torch.optim.SGD(m.parameters(), lr=0.1), 12)
    assert resolve_checkpoint(str(tmp_dir))[1] == 12
    assert resolve_checkpoint(str(tmp_dir / "model_step_12.safetensors"))[1] == 12
