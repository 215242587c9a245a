"""Decode throughput of the 412M model over the latent KV cache.

``python inference/bench_decode.py [--batch 1 32 64] [--prompt 128] [--new 128]
[--impl ours|reference]`` prefills a batch of uniform-random prompts, then
decodes ``--new`` tokens greedily and reports decode tokens/s (device time of
the decode loop, CUDA events; prefill excluded) per batch size as one JSON
line.  Random-init weights of the 412M yaml dims; bf16 compute.

``--impl reference`` runs the reference's own ``Transformer.generate``
(installed in ``baseline/_ref``) under bf16 autocast on the same shapes.
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


def _timed(fn):
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    out = fn()
    b.record()
    torch.cuda.synchronize()
    return out, a.elapsed_time(b)


def run(impl: str, batches, prompt: int, new: int):
    if impl == "reference":
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        cfg_path = ROOT / "baseline" / "_ref" / "configs" / "pretrain_a100_422m.yaml"
    else:
        sys.path.insert(0, str(HERE.parent))
        cfg_path = HERE.parent / "configs" / "pretrain_412m.yaml"
    from models.transformer import Transformer
    cfg = yaml.safe_load(open(cfg_path))["model"]
    torch.manual_seed(0)
    model = Transformer(cfg).cuda().eval()
    res = {}
    for B in batches:
        g = torch.Generator(device="cuda").manual_seed(B)
        p = torch.randint(0, cfg["vocab_size"], (B, prompt), device="cuda", generator=g)
        ctx = torch.autocast("cuda", dtype=torch.bfloat16) if impl == "reference" else torch.no_grad()
        with ctx, torch.inference_mode():
            # warm-up (allocations, weight caches)
            model.generate(p, max_new_tokens=4, temperature=0.0)
            _, t_pre = _timed(lambda: model.generate(p, max_new_tokens=0, temperature=0.0))
            out, t_all = _timed(lambda: model.generate(p, max_new_tokens=new, temperature=0.0))
        n_new = out.shape[1] - prompt
        decode_ms = max(t_all - t_pre, 1e-3)
        res[str(B)] = {"decode_tokens_per_s": round(B * n_new / (decode_ms / 1000.0), 1),
                       "ms_per_token_step": round(decode_ms / max(n_new, 1), 3), "prefill_ms": round(t_pre, 2)}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 32, 64])
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    a = ap.parse_args()
    res = run(a.impl, a.batch, a.prompt, a.new)
    print(json.dumps({"metric": "decode tokens/s (greedy, device time, prefill excluded)", "impl": a.impl,
                      "model": "412m yaml dims, random init", "prompt": a.prompt, "new_tokens": a.new,
                      "results": res}))


if __name__ == "__main__":
    main()
