"""MLA attention microbenchmark: one attention layer at DeepSeek-V3 head dims.

``python -m ops.bench_mla [--impl ours|reference]`` (from
``deepseek-v3-lite_b200/``; ``reference`` needs the reference installed in
``baseline/_ref``) times, on one GPU with CUDA events after warm-up:

prefill  forward + backward of a Multi-Head Latent Attention layer (model
         dim 2048, 16 heads, qk_nope 128 + qk_rope 64, v_head 128,
         kv_lora_rank 512, no q LoRA), batch 8 x 4096 tokens, causal, bf16:
         q / kv_a projections, latent RMSNorm, kv_b up-projection, RoPE,
         attention, o-projection and every gradient;
decode   one new token for each of 64 sequences over a latent cache holding
         4096 positions (absorbed attention over the cache for ours; the
         reference's own stock ``sdpa`` decode path, which re-expands the
         cache through kv_b every step).

Inputs and cache contents are N(0, 1); weights use each module's own init.
``ours`` runs the training engine's MLA forward / backward (tcgen05 GEMMs +
flash attention kernels) and the inference engine's absorbed latent decode;
``reference`` runs the reference's ``MultiHeadLatentAttention`` module
(models/mla.py:14-180 of the reference tree) under bf16 autocast
(prefill) / in bf16 (decode).  Reported FLOP/s count the attention core only
(causal: half of the S x S score matrix), 2.5x the forward for the backward.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
CFG = {
    "vocab_size": 1024, "dim": 2048, "n_layers": 1, "n_heads": 16, "n_dense_layers": 1,
    "n_routed_experts": 8, "n_shared_experts": 1, "n_activated_experts": 2, "inter_dim": 512,
    "moe_inter_dim": 128, "kv_lora_rank": 512, "q_lora_rank": 0, "qk_nope_head_dim": 128,
    "qk_rope_head_dim": 64, "v_head_dim": 128, "max_seq_len": 4096, "rope_theta": 10000,
    "rope_factor": 1.0, "mscale": 1.0, "attn_impl": "sdpa", "weight_tying": False,
}
B_PRE, S_PRE, B_DEC, CTX = 8, 4096, 64, 4096


def _attn_flops(B, H, S, dqk, dv):
    return 2.0 * B * H * S * S / 2 * (dqk + dv)


def _time(fn, warmup=3, iters=10):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def run_ours():
    sys.path.insert(0, str(HERE.parent))
    from models.transformer import Transformer
    from ops.engine import TrainEngine
    from ops.infer import InferenceEngine
    from training.pretrain import TrainingConfig, _unique_params
    dev = torch.device("cuda")
    torch.manual_seed(0)
    model = Transformer(dict(CFG)).to(dev)
    params = _unique_params(model)
    groups = [{"params": [p for p in params if p.dim() >= 2], "weight_decay": 0.1},
              {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0}]
    eng = TrainEngine(model, None, TrainingConfig(lr=1e-4), groups)
    attn = model.layers[0].attn
    wo = attn.wo.weight
    C = eng.C
    T, D = B_PRE * S_PRE, CFG["dim"]
    g = torch.Generator(device="cuda").manual_seed(1)
    xn = torch.randn(T, D, device=dev, generator=g).bfloat16()
    resid = torch.randn(T, D, device=dev, generator=g)
    dres = (torch.randn(T, D, device=dev, generator=g) * 0.01).bfloat16()

    def fwd():
        actx = eng._mla_fwd(attn, xn, B_PRE, S_PRE)
        out = torch.empty_like(resid)
        C.linear_fwd(actx.O, eng.w(wo), out, True, resid)
        return actx

    def fwd_bwd():
        actx = fwd()
        dxn = torch.empty(T, D, device=dev)
        eng._mla_bwd(attn, actx, dres, dxn, B_PRE, S_PRE)

    t_f = _time(fwd)
    t_fb = _time(fwd_bwd)
    dqk = CFG["qk_nope_head_dim"] + CFG["qk_rope_head_dim"]
    fl = _attn_flops(B_PRE, CFG["n_heads"], S_PRE, dqk, CFG["v_head_dim"])
    del eng
    torch.cuda.empty_cache()

    # decode: absorbed attention over a filled latent cache
    inf = InferenceEngine(model)
    attn._ensure_cache(B_DEC, dev, torch.bfloat16)
    gd = torch.Generator(device="cuda").manual_seed(2)
    attn.kv_cache[:B_DEC, :CTX].copy_(torch.randn(B_DEC, CTX, CFG["kv_lora_rank"], device=dev, generator=gd))
    attn.pe_cache[:B_DEC, :CTX].copy_(torch.randn(B_DEC, CTX, CFG["qk_rope_head_dim"], device=dev, generator=gd))
    x1 = torch.randn(B_DEC, D, device=dev, generator=gd).bfloat16()
    pos = torch.full((B_DEC,), CTX - 1, dtype=torch.int32, device=dev)
    out1 = torch.zeros(B_DEC, D, device=dev)

    def dec():
        with torch.no_grad():
            inf._attn_latent(attn, x1, B_DEC, 1, pos, out1)
    t_d = _time(dec, 5, 50)
    return t_f, t_fb, fl, t_d


def run_reference():
    root = HERE.parent.parent / "baseline" / "_ref"
    if not (root / "models" / "mla.py").exists():
        return None
    sys.path.insert(0, str(root))
    from models.mla import MultiHeadLatentAttention  # the reference's own module
    dev = torch.device("cuda")
    torch.manual_seed(0)
    attn = MultiHeadLatentAttention(dict(CFG)).to(dev)
    T, D = B_PRE * S_PRE, CFG["dim"]
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(B_PRE, S_PRE, D, device=dev, generator=g)
    dres = torch.randn(B_PRE, S_PRE, D, device=dev, generator=g) * 0.01
    q = torch.arange(S_PRE, device=dev)[:, None]
    k = torch.arange(S_PRE, device=dev)[None, :]
    mask = torch.where(q >= k, torch.zeros((), device=dev), torch.full((), float("-inf"), device=dev))[None, None]

    def fwd():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            return attn(x, start_pos=0, mask=mask, use_cache=False)

    def fwd_bwd():
        xx = x.detach().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = attn(xx, start_pos=0, mask=mask, use_cache=False)
        out.backward(dres)

    with torch.no_grad():
        t_f = _time(fwd)
    t_fb = _time(fwd_bwd)
    dqk = CFG["qk_nope_head_dim"] + CFG["qk_rope_head_dim"]
    fl = _attn_flops(B_PRE, CFG["n_heads"], S_PRE, dqk, CFG["v_head_dim"])
    attn.zero_grad(set_to_none=True)
    torch.cuda.empty_cache()

    attn = attn.to(torch.bfloat16)
    attn._ensure_cache(B_DEC, dev, torch.bfloat16)
    gd = torch.Generator(device="cuda").manual_seed(2)
    attn.kv_cache[:B_DEC, :CTX].copy_(torch.randn(B_DEC, CTX, CFG["kv_lora_rank"], device=dev, generator=gd))
    attn.pe_cache[:B_DEC, :CTX].copy_(torch.randn(B_DEC, CTX, CFG["qk_rope_head_dim"], device=dev, generator=gd))
    x1 = torch.randn(B_DEC, 1, D, device=dev, generator=gd).bfloat16()

    def dec():
        with torch.no_grad():
            attn(x1, start_pos=CTX - 1, mask=None, use_cache=True)
    t_d = _time(dec, 2, 10)
    return t_f, t_fb, fl, t_d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    a = ap.parse_args()
    res = run_ours() if a.impl == "ours" else run_reference()
    if res is None:
        print(json.dumps({"impl": a.impl, "unavailable": "reference not installed in baseline/_ref"}))
        return
    t_f, t_fb, fl, t_d = res
    cache_bytes = B_DEC * CTX * (CFG["kv_lora_rank"] + CFG["qk_rope_head_dim"]) * 2
    print(json.dumps({
        "metric": "MLA attention layer (device ms)", "impl": a.impl,
        "config": "D2048 H16 qk 128+64 v128 kv_lora 512, bf16, causal",
        "prefill_B8_S4096": {"fwd_ms": round(t_f, 3), "fwd_bwd_ms": round(t_fb, 3),
                             "attn_fwd_tflops": round(fl / t_f / 1e9, 1),
                             "attn_fwd_bwd_tflops": round(3.5 * fl / t_fb / 1e9, 1)},
        "decode_B64_ctx4096": {"ms_per_step": round(t_d, 4), "tokens_per_s": round(B_DEC / (t_d / 1e3), 1),
                               "latent_cache_GBps": round(cache_bytes / (t_d / 1e3) / 1e9, 1)},
    }), flush=True)


if __name__ == "__main__":
    main()
