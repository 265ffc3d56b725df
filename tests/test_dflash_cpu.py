"""DFlash draft model on CPU: the block-causal mask equals the causal mask,
and the fused (chunked LM-head) loss equals a plain PyTorch restatement with
an explicit mask and full logits; the spec-distill trainer steps with it."""

import math

import torch
import torch.nn.functional as F

from lumenrl_b200.models.dflash import DFlashModel, block_causal_mask


def _plain(model, hs, lm, mask, ids, gamma):
    x = torch.cat(hs, -1)
    x = model.input_norm(model.layer_proj(x))
    B, T, D = x.shape
    allowed = block_causal_mask(T, model.block_size)
    for blk in model.blocks:
        h = blk.attn_norm(x)
        q, k, v = blk.qkv(h).view(B, T, 3, blk.heads, D // blk.heads).permute(2, 0, 3, 1, 4)
        s = (q @ k.transpose(-1, -2)) / math.sqrt(D // blk.heads)
        a = torch.softmax(s.masked_fill(~allowed, float("-inf")), -1) @ v
        x = x + blk.out(a.transpose(1, 2).reshape(B, T, D))
        h = blk.ffn_norm(x)
        x = x + blk.w2(F.silu(blk.w1(h)) * blk.w3(h))
    logits = model.out_norm(x) @ lm.t()
    tgt = ids[:, 1: T + 1]
    ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1), reduction="none").view(B, T)
    w = mask * torch.exp(-torch.arange(T, dtype=torch.float32) / gamma)
    acc = ((logits.argmax(-1) == tgt).float() * mask).sum() / mask.sum()
    return (ce * w).sum() / w.sum(), acc


def test_block_causal_is_causal():
    assert torch.equal(block_causal_mask(19, 8), torch.tril(torch.ones(19, 19, dtype=torch.bool)))


def test_dflash_loss_matches_plain_formulation():
    torch.manual_seed(0)
    B, T, D, V, K = 2, 24, 64, 97, 2
    m = DFlashModel(D, num_target_layers=K, num_heads=4, num_layers=2)
    hs = [torch.randn(B, T, D) for _ in range(K)]
    lm = torch.randn(V, D) * 0.1
    ids = torch.randint(0, V, (B, T + 1))
    mask = (torch.rand(B, T) > 0.2).float()
    out = m(hs, lm, mask, ids, loss_decay_gamma=5.0)
    ref_loss, ref_acc = _plain(m, hs, lm, mask, ids, 5.0)
    assert torch.allclose(out["loss"], ref_loss, atol=1e-5, rtol=1e-5)
    assert torch.allclose(out["accuracy"], ref_acc)
    assert out["logits"].shape == (B, T, V)
    # gradients flow to every draft parameter
    out["loss"].backward()
    assert all(p.grad is not None for p in m.parameters())


def test_spec_distill_dflash_step():
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.parallel.dist import ParallelState
    from lumenrl_b200.trainer.spec_distill_trainer import SpecDistillSpec, SpecDistillTrainer
    spec = SpecDistillSpec(aux_layers=(0, 1, 2), seq_len=32, batch_per_rank=2, draft_type="dflash",
                           num_target_layers=2, draft_layers=1)
    tr = SpecDistillTrainer(tiny_qwen3(layers=4), spec, ParallelState())
    first = tr.step()
    for _ in range(3):
        last = tr.step(ids=None)
    assert math.isfinite(first["loss"]) and math.isfinite(last["loss"]) and len(last["acc"]) == 1
