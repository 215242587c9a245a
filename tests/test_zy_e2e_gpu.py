"""End to end on one B200, the way a user runs it: a token shard from the
shard builder -> the trainer's own loop (DataLoader, micro-batches,
optimizer steps, periodic and final checkpoints) -> a fresh model loaded
from the checkpoint directory -> greedy generation, batch-1 speculative
decoding with the checkpoint's MTP head, and batched speculative decoding."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

CFG = {
    "vocab_size": 512, "dim": 256, "n_layers": 3, "n_heads": 4, "n_dense_layers": 1,
    "n_routed_experts": 8, "n_shared_experts": 1, "n_activated_experts": 2, "inter_dim": 512,
    "moe_inter_dim": 128, "kv_lora_rank": 64, "q_lora_rank": 0, "qk_nope_head_dim": 48,
    "qk_rope_head_dim": 16, "v_head_dim": 64, "max_seq_len": 128, "rope_theta": 10000,
    "rope_factor": 1.0, "mscale": 1.0, "mtp_depth": 1, "mtp_loss_weight": 0.3,
    "attn_impl": "sdpa", "weight_tying": True,
}


def _eager_loss(model, batch):
    model.eval()
    with torch.no_grad():
        logits = model(batch[:, :-1], start_pos=0, use_cache=False)
        loss = F.cross_entropy(logits.float().flatten(0, 1), batch[:, 1:].flatten()).item()
    model.train()
    return loss


def test_shard_train_resume_decode(tmp_path):
    from data.build_small_shard import build_shard, open_source, open_tokenizer
    from inference.generate import load_mtp_draft, resolve_checkpoint
    from inference.speculative import BatchedSpeculativeDecoder, SpeculativeDecoder
    from models.transformer import Transformer
    from training.pretrain import PretrainDataset, Pretrainer, TrainingConfig

    encode, eos, vocab = open_tokenizer("bytes")
    assert vocab <= CFG["vocab_size"]
    build_shard(str(tmp_path / "data"), open_source("synthetic"), encode, eos, target_tokens=80_000)
    held_out = torch.stack([torch.cat(PretrainDataset(str(tmp_path / "data"), 128, vocab)[i]) for i in (1, 5, 9, 13)])
    held_out = torch.cat([held_out[:, :128], held_out[:, -1:]], dim=1).long().cuda()

    cfg = TrainingConfig(model_config=dict(CFG), data_path=str(tmp_path / "data"),
                         checkpoint_dir=str(tmp_path / "ckpt"), max_seq_len=128, vocab_size=CFG["vocab_size"],
                         batch_size=8, gradient_accumulation_steps=2, max_steps=60, warmup_steps=4, lr=3e-3,
                         mtp_weight=0.3, save_every=30, log_every=20, log_per_component_params=False,
                         compile_model=False, grad_checkpoint=False)
    tr = Pretrainer(cfg)
    before = _eager_loss(tr.raw_model, held_out)
    tr.train()
    after = _eager_loss(tr.raw_model, held_out)
    tr.engine.check()
    assert after < before - 1.0, (before, after)
    mgr, step = resolve_checkpoint(str(tmp_path / "ckpt"))
    assert step == 60 and 30 in mgr._list_steps()

    model = Transformer(dict(CFG)).cuda()
    mgr.load(model, step, device="cuda", strict=False)
    model.eval()
    assert abs(_eager_loss(model, held_out) - after) < 1e-3
    prompt = held_out[:1, :32]
    with torch.inference_mode():
        greedy = model.generate(prompt, max_new_tokens=24, temperature=0.0)
    assert greedy.shape[1] == 32 + 24 and int(greedy.max()) < CFG["vocab_size"]
    mtp = load_mtp_draft(model, dict(CFG), mgr, step, "cuda")
    with torch.inference_mode():
        spec = SpeculativeDecoder(model, mtp).generate(prompt, max_new_tokens=24, temperature=0.0)
    assert spec.shape[1] >= 32 + 24
    # greedy speculative decoding keeps exactly the main model's tokens
    assert torch.equal(spec[:, :32 + 24], greedy)
    toks, lengths = BatchedSpeculativeDecoder(model, mtp).generate(held_out[:4, :32], max_new_tokens=16)
    assert bool((lengths >= 32 + 16).all())
    assert torch.equal(toks[0, :32 + 16], greedy[0, :32 + 16])
    tr.engine.close()
