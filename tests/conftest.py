"""Shared pytest setup: import path, the ``gpu`` marker and small configs."""
import os
import shutil
import sys
import tempfile
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "deepseek-v3-lite_b200"
if str(SRC) not in sys.path:
    sys.path.insert(0, str(SRC))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def small_cfg():
    return {
        "vocab_size": 1024, "dim": 64, "n_layers": 2, "n_heads": 4, "n_dense_layers": 1,
        "n_routed_experts": 4, "n_shared_experts": 1, "n_activated_experts": 2, "inter_dim": 128,
        "moe_inter_dim": 64, "kv_lora_rank": 16, "q_lora_rank": 0, "qk_nope_head_dim": 8,
        "qk_rope_head_dim": 4, "v_head_dim": 8, "max_seq_len": 64, "rope_theta": 10000,
        "rope_factor": 1.0, "mscale": 1.0, "mtp_depth": 1, "mtp_loss_weight": 0.3,
        "attn_impl": "sdpa", "weight_tying": True,
    }


@pytest.fixture(scope="session")
def mid_cfg():
    """Wider config (vocab 100018 like the 412M model, 2 layers)."""
    return {
        "vocab_size": 100018, "dim": 256, "n_layers": 2, "n_heads": 4, "n_dense_layers": 1,
        "n_routed_experts": 8, "n_shared_experts": 1, "n_activated_experts": 2, "inter_dim": 512,
        "moe_inter_dim": 128, "kv_lora_rank": 64, "q_lora_rank": 0, "qk_nope_head_dim": 48,
        "qk_rope_head_dim": 16, "v_head_dim": 64, "max_seq_len": 128, "rope_theta": 10000,
        "rope_factor": 1.0, "mscale": 1.0, "mtp_depth": 1, "mtp_loss_weight": 0.3,
        "attn_impl": "sdpa", "weight_tying": True,
    }


@pytest.fixture()
def tmp_dir():
    d = Path(tempfile.mkdtemp(prefix="dsv3_test_"))
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture()
def token_file(tmp_dir):
    data = torch.randint(0, 1024, (512,), dtype=torch.long)
    path = tmp_dir / "tokens.bin"
    torch.save(data, path)
    return str(path)


@pytest.fixture()
def shard_dir(tmp_dir):
    d = tmp_dir / "shards"
    d.mkdir()
    for i in range(3):
        torch.save(torch.arange(i * 128, (i + 1) * 128, dtype=torch.long), d / f"shard_{i:05d}.bin")
    return str(d)
