"""Interactive generation CLI (cached decode, optional MTP speculative decoding).

Same flags and flow as the reference (``inference/generate.py:22-123``):
``--config --checkpoint --max_new_tokens --temperature --top_p
--use_speculative --acceptance_threshold --device``.  A checkpoint directory
resolves to its latest complete step; a file path resolves to the step in its
name.  MTP draft weights are the ``mtp.``-prefixed keys of the checkpoint.
"""
from __future__ import annotations

import os
import sys
from argparse import ArgumentParser
from pathlib import Path
from typing import Optional

import torch
import yaml

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from inference.speculative import SpeculativeDecoder  # noqa: E402
from models.mtp import MTPModule  # noqa: E402
from models.transformer import Transformer  # noqa: E402
from utils.checkpoint import CheckpointManager  # noqa: E402

try:
    from transformers import AutoTokenizer
    HAS_TRANSFORMERS = True
except ImportError:  # decode helpers still work without a tokenizer
    AutoTokenizer = None
    HAS_TRANSFORMERS = False


def load_config(path: str) -> dict:
    """Load a YAML config that must contain a ``model`` section."""
    if not os.path.exists(path):
        raise FileNotFoundError(f"Config not found: {path}")
    with open(path) as f:
        cfg = yaml.safe_load(f)
    if not isinstance(cfg, dict) or "model" not in cfg:
        raise ValueError("Config must be a dict with a 'model' section")
    return cfg


def resolve_checkpoint(path: str):
    """``(CheckpointManager, step)`` for a checkpoint directory or weight file."""
    ckpt_dir = path if os.path.isdir(path) else str(Path(path).parent)
    mgr = CheckpointManager(ckpt_dir)
    if os.path.isdir(path):
        step = mgr.latest_step()
        if step is None:
            raise RuntimeError(f"No checkpoints found in {ckpt_dir}")
        return mgr, step
    tail = Path(path).stem.rsplit("_", 1)[-1]
    return mgr, int(tail) if tail.isdigit() else mgr.latest_step()


def load_mtp_draft(model: Transformer, model_cfg: dict, mgr: CheckpointManager, step: int, device) -> MTPModule:
    """Depth-1 MTP module with the checkpoint's ``mtp.mtp_modules.0.*`` weights."""
    mtp = MTPModule(model_cfg, depth=1).to(device).eval()
    mtp.set_output_head(model.head)
    wpath = mgr.save_dir / f"model_step_{step}.safetensors"
    if wpath.exists():
        from safetensors.torch import load_file
        prefix = "mtp.mtp_modules.0."
        state = {k[len(prefix):]: v for k, v in load_file(str(wpath), device=str(device)).items() if k.startswith(prefix)}
        if state:
            mtp.load_state_dict(state, strict=False)
            print("MTP weights loaded.")
        else:
            print("[warn] No MTP weights in checkpoint; draft head is uninitialised.")
    return mtp


@torch.inference_mode()
def generate_interactive(model: torch.nn.Module, tokenizer, args, mtp_module: Optional[MTPModule] = None) -> None:
    """Chat REPL: ``/exit`` quits, ``/clear`` resets the conversation."""
    print("DeepSeek-V3-Lite  |  /exit to quit  |  /clear to reset context")
    history = []
    decoder = None
    if mtp_module is not None and args.use_speculative:
        decoder = SpeculativeDecoder(model, mtp_module, acceptance_threshold=args.acceptance_threshold)
        print("Speculative decoding enabled.")
    while True:
        try:
            text = input("\n>>> ").strip()
        except (EOFError, KeyboardInterrupt):
            print("\nExiting.")
            break
        if text == "/exit":
            break
        if text == "/clear":
            history.clear()
            print("[context cleared]")
            continue
        if not text:
            continue
        history.append({"role": "user", "content": text})
        ids = tokenizer.apply_chat_template(history, add_generation_prompt=True, return_tensors="pt").to(args.device)
        if decoder is not None:
            out = decoder.generate(ids, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                                   eos_token_id=tokenizer.eos_token_id)
        else:
            out = model.generate(ids, max_new_tokens=args.max_new_tokens, temperature=args.temperature,
                                 top_p=args.top_p, eos_token_id=tokenizer.eos_token_id)
        reply = tokenizer.decode(out[0, ids.shape[1]:], skip_special_tokens=True)
        print(f"\nAssistant: {reply}")
        history.append({"role": "assistant", "content": reply})


def main() -> None:
    if not HAS_TRANSFORMERS:
        raise RuntimeError("`transformers` is required for the interactive CLI.")
    ap = ArgumentParser(description="Run DeepSeek-V3-Lite inference")
    ap.add_argument("--config", type=str, required=True)
    ap.add_argument("--checkpoint", type=str, required=True)
    ap.add_argument("--max_new_tokens", type=int, default=512)
    ap.add_argument("--temperature", type=float, default=0.7)
    ap.add_argument("--top_p", type=float, default=0.9)
    ap.add_argument("--use_speculative", action="store_true")
    ap.add_argument("--acceptance_threshold", type=float, default=0.8)
    ap.add_argument("--device", type=str, default="cuda" if torch.cuda.is_available() else "cpu")
    args = ap.parse_args()
    cfg = load_config(args.config)
    model = Transformer(cfg["model"]).to(args.device).eval()
    mgr, step = resolve_checkpoint(args.checkpoint)
    print(f"Loading checkpoint step {step}...")
    mgr.load(model, step, device=args.device, strict=False)
    mtp = load_mtp_draft(model, cfg["model"], mgr, step, args.device) if args.use_speculative else None
    tok_path = cfg.get("data", {}).get("tokenizer_path", "deepseek-ai/deepseek-coder-v2-lite")
    tokenizer = AutoTokenizer.from_pretrained(tok_path)
    generate_interactive(model, tokenizer, args, mtp)


if __name__ == "__main__":
    main()
