"""Tiny-config smoke benchmark (B1): one training step and a short greedy decode.

``python training/bench_tiny.py [--impl ours|reference] [--steps 5] [--new 16]``
(from ``deepseek-v3-lite_b200/``) measures the workload of the suite's tiny
baseline: the ~2M-parameter config with every feature on (MLA, MoE with a
shared expert, aux-loss-free bias, MTP at weight 0.3, tied head), batch
4 x 128 uniform tokens (seed 0), forward + backward + AdamW; the median of
``--steps`` steps after one warm-up step; then greedy generation of ``--new``
tokens from a 16-token prompt at batch 1.  CUDA events on a GPU,
``time.perf_counter`` on the CPU.

ours       ``configs/pretrain_tiny.yaml`` through this package's Pretrainer
           (the native engine on CUDA, PyTorch on the CPU) and
           ``Transformer.generate``;
reference  the reference's own Pretrainer and Transformer from
           ``baseline/_ref`` on its ``configs/pretrain_1650_2m.yaml`` (the
           same dims), without ``torch.compile``.

Prints one JSON line.  Run it as a script (not ``-m``): the two arms import
different packages under the same top-level names.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import tempfile
import time
from pathlib import Path

import torch
import yaml

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent


class _Timer:
    def __init__(self, device):
        self.cuda = device.type == "cuda"

    def __call__(self, fn):
        if self.cuda:
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            torch.cuda.synchronize()
            a.record()
            out = fn()
            b.record()
            torch.cuda.synchronize()
            return out, a.elapsed_time(b)
        t0 = time.perf_counter()
        out = fn()
        return out, (time.perf_counter() - t0) * 1e3


def _positive(v: str) -> int:
    n = int(v)
    if n < 1:
        raise argparse.ArgumentTypeError("--steps must be at least 1")
    return n


def _measure(trainer, model, vocab, steps, new, device):
    timer = _Timer(device)
    g = torch.Generator().manual_seed(0)
    tok = torch.randint(0, vocab, (4, 129), generator=g).to(device)
    trainer.train_step(tok[:, :-1], tok[:, 1:], 0)                       # warm-up
    times, last = [], None
    for i in range(steps):
        out, ms = timer(lambda: trainer.train_step(tok[:, :-1], tok[:, 1:], i + 1))
        times.append(ms)
        if out is not None:          # None: the NaN guard skipped this micro-batch
            last = out
    loss = float(last["loss"]) if last is not None else None
    step_ms = statistics.median(times)
    prompt = torch.randint(0, vocab, (1, 16), generator=g).to(device)
    model.eval()
    with torch.no_grad():
        model.generate(prompt, max_new_tokens=2, temperature=0.0)      # warm-up
        gen, dec_ms = timer(lambda: model.generate(prompt, max_new_tokens=new, temperature=0.0))
    produced = int(gen.shape[1] - prompt.shape[1])
    return {"step_ms": round(step_ms, 3), "train_tokens_per_s": round(4 * 128 / (step_ms / 1e3), 1),
            "last_loss": round(loss, 4) if loss is not None else None, "decode_ms": round(dec_ms, 3), "decode_tokens": produced,
            "decode_tokens_per_s": round(produced / (dec_ms / 1e3), 1)}


def run_ours(steps, new, device):
    sys.path.insert(0, str(PKG))
    from training.pretrain import Pretrainer, config_from_yaml
    y = yaml.safe_load(open(PKG / "configs" / "pretrain_tiny.yaml"))
    cfg = config_from_yaml(y, checkpoint_dir=tempfile.mkdtemp(prefix="dsv3_tiny_"))
    cfg.batch_size, cfg.gradient_accumulation_steps, cfg.mtp_weight = 4, 1, 0.3
    cfg.max_seq_len, cfg.warmup_steps, cfg.max_steps = 128, 1, 10 ** 6
    cfg.log_per_component_params = False
    tr = Pretrainer(cfg)
    res = _measure(tr, tr.raw_model, y["model"]["vocab_size"], steps, new, tr.device)
    if tr.engine is not None:
        tr.engine.check()
        tr.engine.close()
    return res


def run_reference(steps, new, device):
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "training" / "pretrain.py").exists():
        return None
    sys.path.insert(0, str(ref))
    from training.pretrain import Pretrainer, TrainingConfig   # the reference's own trainer
    y = yaml.safe_load(open(ref / "configs" / "pretrain_1650_2m.yaml"))
    m = y["model"]
    cfg = TrainingConfig(model_config=y, data_path="/nonexistent", checkpoint_dir=tempfile.mkdtemp(prefix="ref_tiny_"),
                         max_seq_len=128, vocab_size=m["vocab_size"], batch_size=4, gradient_accumulation_steps=1,
                         max_steps=10 ** 6, warmup_steps=1, compile_model=False, mtp_weight=0.3,
                         log_per_component_params=False)
    tr = Pretrainer(cfg)
    return _measure(tr, tr.raw_model, m["vocab_size"], steps, new, tr.device)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--steps", type=_positive, default=5)
    ap.add_argument("--new", type=int, default=16)
    a = ap.parse_args(argv)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    res = run_ours(a.steps, a.new, device) if a.impl == "ours" else run_reference(a.steps, a.new, device)
    line = {"metric": "tiny config: train step ms (batch 4 x 128, fwd+bwd+AdamW, MTP) and greedy decode tokens/s",
            "impl": a.impl, "device": device.type}
    line.update(res if res is not None else {"unavailable": "reference not installed in baseline/_ref"})
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
