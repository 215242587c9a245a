"""MTP speculative decoding throughput of the scaled model (random init).

``python inference/bench_spec.py [--config configs/scaled_13b.yaml]
[--batch 32] [--prompt 128] [--new 128] [--impl ours|reference]`` builds the
model (~14B parameters with the MTP head) directly on the GPU, prefills
uniform-random prompts and times the decode loop with CUDA events (prefill
excluded):

ours       ``BatchedSpeculativeDecoder``: all rows per step (native
           absorbed-MLA decode step from a CUDA graph, grouped expert GEMMs,
           per-row acceptance, per-row cache positions);
reference  the reference's ``SpeculativeDecoder``, which is batch-1 only, run
           on ``--ref-rows`` of the prompts one after another under bf16
           autocast (tokens/s of that sequential run; the rate of 32
           sequential runs is the same).

Tokens/s counts every generated token (main + accepted drafts).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch
import yaml

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def _events():
    return torch.cuda.Event(True), torch.cuda.Event(True)


def run_ours(cfg, batch, prompt, new):
    sys.path.insert(0, str(HERE.parent))
    from inference.speculative import BatchedSpeculativeDecoder
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Transformer(dict(cfg))
        mtp = MultiTokenPrediction(dict(cfg), model)
    model.eval()
    mtp.eval()
    dec = BatchedSpeculativeDecoder(model, mtp.mtp_modules[0])
    g = torch.Generator(device="cuda").manual_seed(1)
    p = torch.randint(0, cfg["vocab_size"], (batch, prompt), device="cuda", generator=g)
    dec.generate(p, max_new_tokens=4)                     # warm-up: weight caches, graphs
    a, b = _events()
    with torch.inference_mode():
        model.reset_cache()
        a.record()
        model(p, start_pos=0, use_cache=True)
        b.record()
    torch.cuda.synchronize()
    t_pre = a.elapsed_time(b)
    a.record()
    buf, lengths = dec.generate(p, max_new_tokens=new)
    b.record()
    torch.cuda.synchronize()
    t_all = a.elapsed_time(b)
    produced = int((lengths - prompt).sum().item())
    decode_ms = max(t_all - t_pre, 1e-3)
    return {"rows": batch, "decode_ms": round(decode_ms, 2), "tokens": produced,
            "tokens_per_s": round(produced / (decode_ms / 1e3), 1), "mean_tokens_per_row": round(produced / batch, 1)}


def run_reference(cfg, rows, prompt, new):
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "inference" / "speculative.py").exists():
        return None
    sys.path.insert(0, str(ref))
    from inference.speculative import SpeculativeDecoder  # the reference's own decoder
    from models.mtp import MultiTokenPrediction
    from models.transformer import Transformer
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Transformer(dict(cfg))
        mtp = MultiTokenPrediction(dict(cfg), model)
    model.eval()
    mtp.eval()
    dec = SpeculativeDecoder(model, mtp.mtp_modules[0])
    g = torch.Generator(device="cuda").manual_seed(1)
    p = torch.randint(0, cfg["vocab_size"], (rows, prompt), device="cuda", generator=g)
    produced, decode_ms = 0, 0.0
    with torch.autocast("cuda", dtype=torch.bfloat16), torch.inference_mode():
        dec.generate(p[:1], max_new_tokens=2)             # warm-up
        for r in range(rows):
            a, b = _events()
            model.reset_cache()
            a.record()
            model(p[r:r + 1], start_pos=0, use_cache=True)
            b.record()
            torch.cuda.synchronize()
            t_pre = a.elapsed_time(b)
            a.record()
            out = dec.generate(p[r:r + 1], max_new_tokens=new)
            b.record()
            torch.cuda.synchronize()
            decode_ms += max(a.elapsed_time(b) - t_pre, 1e-3)
            produced += out.shape[1] - prompt
    return {"rows": rows, "sequential": True, "decode_ms": round(decode_ms, 2), "tokens": produced,
            "tokens_per_s": round(produced / (decode_ms / 1e3), 1), "mean_tokens_per_row": round(produced / rows, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=str(HERE.parent / "configs" / "scaled_13b.yaml"))
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--ref-rows", type=int, default=2, help="prompts the batch-1 reference decodes one by one")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    a = ap.parse_args()
    cfg = yaml.safe_load(open(a.config))["model"]
    res = run_ours(cfg, a.batch, a.prompt, a.new) if a.impl == "ours" else run_reference(cfg, a.ref_rows, a.prompt,
                                                                                          a.new)
    line = {"metric": "MTP speculative decode tokens/s (device time, prefill excluded)", "impl": a.impl,
            "model": Path(a.config).stem + " (random init)", "prompt": a.prompt, "new_tokens": a.new}
    line.update(res if res is not None else {"unavailable": "reference not installed in baseline/_ref"})
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
