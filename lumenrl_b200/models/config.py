"""Model architecture descriptions and presets.

``ModelArgs`` covers the decoder families the reference trains: Llama-style
(no QK-norm), Qwen3 dense (QK-RMSNorm) and Qwen3-MoE (softmax top-k router,
renormalised).  ``from_hf_config`` reads an HF ``config.json`` dict so a local
checkpoint directory can be loaded.
"""

from __future__ import annotations

from dataclasses import dataclass, field, asdict
from typing import Optional


@dataclass
class ModelArgs:
    vocab_size: int = 151936
    hidden_size: int = 4096
    num_layers: int = 36
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 12288
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    rope_scaling: Optional[dict] = None
    qk_norm: bool = True
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 40960
    init_std: float = 0.02
    # MoE (num_experts == 0 -> dense MLP in every layer)
    num_experts: int = 0
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    norm_topk_prob: bool = True
    router_aux_loss_coef: float = 0.0
    decoder_sparse_step: int = 1
    mlp_only_layers: list = field(default_factory=list)
    name: str = "qwen3"

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i not in self.mlp_only_layers and (i + 1) % self.decoder_sparse_step == 0

    def num_params(self) -> int:
        from lumenrl_b200.models.qwen3 import param_specs
        n = 0
        for _, shape in param_specs(self):
            k = 1
            for s in shape:
                k *= s
            n += k
        return n

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return self.num_layers * 2 * self.kv_dim * dtype_bytes

    def to_dict(self) -> dict:
        return asdict(self)


def qwen3_8b() -> ModelArgs:
    return ModelArgs(name="Qwen3-8B")


def qwen3_30b_a3b() -> ModelArgs:
    return ModelArgs(name="Qwen3-30B-A3B", vocab_size=151936, hidden_size=2048, num_layers=48, num_heads=32,
                     num_kv_heads=4, head_dim=128, intermediate_size=6144, num_experts=128, num_experts_per_tok=8,
                     moe_intermediate_size=768, router_aux_loss_coef=1e-3)


def tiny_llama(vocab: int = 2048) -> ModelArgs:
    """The CPU plumbing model: 2 layers, hidden 256, 4q/2kv heads of 64, SwiGLU
    688, RoPE theta 1e4, tied embeddings, no QK-norm."""
    return ModelArgs(name="tiny-llama", vocab_size=vocab, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                     head_dim=64, intermediate_size=688, rope_theta=10000.0, qk_norm=False, tie_word_embeddings=True,
                     max_position_embeddings=4096)


def tiny_qwen3(vocab: int = 2048, layers: int = 2) -> ModelArgs:
    """Qwen3 block structure at toy size; head_dim 128 like the real model so
    every GPU kernel (decode attention included) runs its production shape."""
    return ModelArgs(name="tiny-qwen3", vocab_size=vocab, hidden_size=256, num_layers=layers, num_heads=4,
                     num_kv_heads=2, head_dim=128, intermediate_size=512, qk_norm=True, max_position_embeddings=4096)


def tiny_qwen3_moe(vocab: int = 2048) -> ModelArgs:
    return ModelArgs(name="tiny-qwen3-moe", vocab_size=vocab, hidden_size=256, num_layers=2, num_heads=4,
                     num_kv_heads=2, head_dim=128, intermediate_size=512, num_experts=8, num_experts_per_tok=2,
                     moe_intermediate_size=128, router_aux_loss_coef=1e-3, max_position_embeddings=4096)


PRESETS = {
    "qwen3-8b": qwen3_8b,
    "Qwen/Qwen3-8B": qwen3_8b,
    "Qwen/Qwen3-8B-Base": qwen3_8b,
    "qwen3-30b-a3b": qwen3_30b_a3b,
    "Qwen/Qwen3-30B-A3B": qwen3_30b_a3b,
    "tiny-llama": tiny_llama,
    "tiny-qwen3": tiny_qwen3,
    "tiny-qwen3-moe": tiny_qwen3_moe,
}


def from_hf_config(cfg: dict) -> ModelArgs:
    moe = int(cfg.get("num_experts", 0) or 0)
    hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    return ModelArgs(
        name=cfg.get("model_type", "qwen3"), vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"],
        num_layers=cfg["num_hidden_layers"], num_heads=cfg["num_attention_heads"],
        num_kv_heads=cfg.get("num_key_value_heads", cfg["num_attention_heads"]), head_dim=hd,
        intermediate_size=cfg.get("intermediate_size", 0), rms_norm_eps=cfg.get("rms_norm_eps", 1e-6),
        rope_theta=cfg.get("rope_theta", 10000.0), rope_scaling=cfg.get("rope_scaling"),
        qk_norm=cfg.get("model_type", "").startswith("qwen3"), tie_word_embeddings=cfg.get("tie_word_embeddings", False),
        max_position_embeddings=cfg.get("max_position_embeddings", 4096), num_experts=moe,
        num_experts_per_tok=cfg.get("num_experts_per_tok", 8), moe_intermediate_size=cfg.get("moe_intermediate_size", 0),
        norm_topk_prob=cfg.get("norm_topk_prob", True), router_aux_loss_coef=cfg.get("router_aux_loss_coef", 0.0),
        decoder_sparse_step=cfg.get("decoder_sparse_step", 1), mlp_only_layers=list(cfg.get("mlp_only_layers", [])))


def resolve_model(name: str) -> ModelArgs:
    """Preset name, or a directory holding an HF ``config.json``."""
    import json
    import os
    if name in PRESETS:
        return PRESETS[name]()
    path = os.path.join(name, "config.json")
    if os.path.isfile(path):
        with open(path) as f:
            return from_hf_config(json.load(f))
    low = name.lower()
    for key, fn in PRESETS.items():
        if key.lower() in low:
            return fn()
    raise KeyError(f"unknown model {name!r}; presets: {sorted(PRESETS)}")
