"""Pre-training data preparation entry point.

The reference (``data/prepare_data.py:23-84``) writes a data config with the
DeepSeek tokenizer identifiers and hands the work to an external corpus
pipeline (``shared_data.prepare_data.run_pipeline``: download, clean,
tokenize, pack into ``shard_*.bin`` files of 50M uint32 tokens).  This module
keeps that interface: it writes ``data/data_config.yaml`` with the same
tokenizer fields and calls the external pipeline when it is installed.
Without it, it says so and points at ``data.build_small_shard``, which writes
a shard of the same format from local or synthetic text.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import yaml

DEEPSEEK_TOKENIZER_NAME = "deepseek-coder-v2-lite"
DEEPSEEK_VOCAB_SIZE = 100_018
DEEPSEEK_EOS_TOKEN_ID = 100_017
DEEPSEEK_PAD_TOKEN_ID = 100_016
SHARD_TOKENS = 50_000_000

_HERE = Path(__file__).resolve().parent


def write_data_config(out_path: Path, base: dict = None) -> Path:
    """``base`` (the external pipeline's universal config, if any) with the
    tokenizer fields set to the DeepSeek values."""
    cfg = dict(base or {})
    pipe = dict(cfg.get("pipeline", {}))
    tok = dict(pipe.get("tokenizer", {}))
    tok.update(name=DEEPSEEK_TOKENIZER_NAME, vocab_size=DEEPSEEK_VOCAB_SIZE, eos_token_id=DEEPSEEK_EOS_TOKEN_ID,
               pad_token_id=DEEPSEEK_PAD_TOKEN_ID)
    pipe["tokenizer"] = tok
    pipe.setdefault("shard_tokens", SHARD_TOKENS)
    cfg["pipeline"] = pipe
    cfg["_generator"] = "deepseek-v3-lite_b200/data/prepare_data.py"
    cfg["_tokenizer_family"] = "deepseek-coder-v2"
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(yaml.safe_dump(cfg, sort_keys=False, allow_unicode=True), encoding="utf-8")
    return out_path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="DeepSeek-v3-Lite data preparation (external corpus pipeline)")
    ap.add_argument("--stage", choices=["pretrain"], default="pretrain")
    ap.add_argument("--mixture", default=None)
    ap.add_argument("--data-config", default=None)
    ap.add_argument("--data-root", default=None)
    ap.add_argument("--source", default=None)
    for flag in ("download", "clean", "tokenize", "pack"):
        ap.add_argument(f"--skip-{flag}", action="store_true")
    ap.add_argument("--config-out", default=str(_HERE / "data_config.yaml"), help="where the data config is written")
    a = ap.parse_args(argv)
    try:
        from shared_data import config as sd_config
        from shared_data.common import load_yaml
        from shared_data.prepare_data import run_pipeline
    except ImportError:
        cfg = write_data_config(Path(a.config_out))
        print(f"[data] wrote {cfg} (tokenizer {DEEPSEEK_TOKENIZER_NAME}, vocab {DEEPSEEK_VOCAB_SIZE:,}, "
              f"EOS {DEEPSEEK_EOS_TOKEN_ID}).\n[data] the external `shared_data` corpus pipeline is not installed; "
              f"build a shard from local or synthetic text with `python -m data.build_small_shard`.")
        return 2
    cfg = write_data_config(Path(a.config_out), load_yaml(sd_config.UNIVERSAL_DATA_CONFIG_PATH))
    return run_pipeline(mixture_path=Path(a.mixture) if a.mixture else sd_config.UNIVERSAL_MIXTURE_PATH,
                        data_config_path=Path(a.data_config) if a.data_config else cfg, source=a.source,
                        skip_download=a.skip_download, skip_clean=a.skip_clean, skip_tokenize=a.skip_tokenize,
                        skip_pack=a.skip_pack, data_root=Path(a.data_root) if a.data_root else None)


if __name__ == "__main__":
    sys.exit(main())
