"""Qwen3 / Llama-style decoder (dense and MoE) over a flat parameter store.

Design (B200-first):

* Every parameter is a view into ONE contiguous bf16 buffer (``FlatParams``).
  The same buffer is the rollout engine's weights (colocated mode), the
  source of weight sync, and the all-gather target of sharded training, so a
  weight update is one fused pass over one allocation.
* Projections are fused: ``wqkv`` = [q; k; v] rows, ``w13`` = [gate; up] rows,
  so each block issues one GEMM per projection group.
* Weight gradients are never materialised in bf16: each weight carries a
  ``main_grad`` view into the flat fp32 gradient buffer and the backward GEMMs
  accumulate into it (beta = 1).

HF names (``model.layers.{i}.self_attn.q_proj.weight`` ...) are produced and
consumed by ``hf_state_dict`` / ``load_hf_state_dict`` so checkpoints stay
safetensors-compatible with the reference's exports
(reference ``lumenrl/workers/actor_worker.py:931-1043``).
"""

from __future__ import annotations

import math
from typing import Iterator, Optional

import torch
import torch.nn as nn
from torch import Tensor
from torch.utils.checkpoint import checkpoint as _ckpt

from lumenrl_b200 import ops
from lumenrl_b200.models.config import ModelArgs

ALIGN = 128  # elements; every tensor in the flat buffer starts 256-byte aligned


def param_specs(a: ModelArgs) -> list[tuple[str, tuple[int, ...]]]:
    H = a.hidden_size
    specs: list[tuple[str, tuple[int, ...]]] = [("embed", (a.vocab_size, H))]
    for i in range(a.num_layers):
        p = f"layers.{i}."
        specs.append((p + "ln1", (H,)))
        specs.append((p + "wqkv", (a.qkv_dim, H)))
        if a.qk_norm:
            specs.append((p + "q_norm", (a.head_dim,)))
            specs.append((p + "k_norm", (a.head_dim,)))
        specs.append((p + "wo", (H, a.q_dim)))
        specs.append((p + "ln2", (H,)))
        if a.is_moe_layer(i):
            E, Fe = a.num_experts, a.moe_intermediate_size
            specs.append((p + "router", (E, H)))
            specs.append((p + "experts_w13", (E, 2 * Fe, H)))
            specs.append((p + "experts_w2", (E, H, Fe)))
        else:
            specs.append((p + "w13", (2 * a.intermediate_size, H)))
            specs.append((p + "w2", (H, a.intermediate_size)))
    specs.append(("norm", (H,)))
    if not a.tie_word_embeddings:
        specs.append(("lm_head", (a.vocab_size, H)))
    return specs


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


class FlatLayout:
    """name -> (offset, shape) inside a flat buffer, each start ALIGN-aligned."""

    def __init__(self, specs: list[tuple[str, tuple[int, ...]]], align: int = ALIGN) -> None:
        self.entries: dict[str, tuple[int, tuple[int, ...]]] = {}
        off = 0
        for name, shape in specs:
            off = (off + align - 1) // align * align
            self.entries[name] = (off, tuple(shape))
            off += _numel(shape)
        self.numel = (off + align - 1) // align * align

    def view(self, flat: Tensor, name: str) -> Tensor:
        off, shape = self.entries[name]
        return flat[off: off + _numel(shape)].view(shape)

    def names(self) -> list[str]:
        return list(self.entries)

    def layer_range(self, layer: int) -> tuple[int, int]:
        """[start, end) of all tensors of one decoder layer (a sync bucket)."""
        keys = [k for k in self.entries if k.startswith(f"layers.{layer}.")]
        lo = min(self.entries[k][0] for k in keys)
        hi = max(self.entries[k][0] + _numel(self.entries[k][1]) for k in keys)
        return lo, hi


def is_matrix(name: str) -> bool:
    return not (name.endswith("ln1") or name.endswith("ln2") or name.endswith("norm") or name.endswith("_norm"))


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w, w_handle):
        ctx.save_for_backward(ids)
        ctx.w_handle, ctx.shape = w_handle, w.shape
        return torch.nn.functional.embedding(ids, w)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        mg = getattr(ctx.w_handle, "main_grad", None)
        if mg is None:
            g = torch.zeros(ctx.shape, dtype=torch.float32, device=dy.device)
            g.index_add_(0, ids.reshape(-1), dy.reshape(-1, dy.shape[-1]).float())
            ops._accum_main_grad(ctx.w_handle, g)
        else:
            mg.index_add_(0, ids.reshape(-1), dy.reshape(-1, dy.shape[-1]).float())
        return None, None, None


def embed(ids: Tensor, w: Tensor) -> Tensor:
    if torch.is_grad_enabled() and w.requires_grad:
        return _Embedding.apply(ids, w.detach(), w)
    return torch.nn.functional.embedding(ids, w)


class Qwen3Model(nn.Module):
    """Decoder with flat storage.  ``forward_packed`` is the training/scoring
    path over packed sequences; the rollout engine drives the same weights
    through ``engine.inference.runner``."""

    def __init__(self, args: ModelArgs, device="cpu", dtype: torch.dtype = torch.bfloat16,
                 flat: Optional[Tensor] = None, requires_grad: bool = True) -> None:
        super().__init__()
        self.args = args
        self.layout = FlatLayout(param_specs(args))
        if flat is None:
            flat = torch.zeros(self.layout.numel, dtype=dtype, device=device)
        if flat.numel() < self.layout.numel:
            raise ValueError("flat buffer too small for the model layout")
        self.flat = flat
        self._params: dict[str, nn.Parameter] = {}
        for name in self.layout.names():
            p = nn.Parameter(self.layout.view(flat, name), requires_grad=requires_grad)
            self._params[name] = p
            self.register_parameter("p__" + name.replace(".", "__"), p)
        self.register_buffer("inv_freq", ops.inv_freq_table(args.head_dim, args.rope_theta, args.rope_scaling,
                                                            flat.device), persistent=False)
        self.gradient_checkpointing = False
        self.recompute_layers: set[int] = set()   # per-layer activation recomputation (memory budget)
        self.routing_replay = None   # set by moe.r3 for rollout routing replay
        self.aux_losses: list[Tensor] = []
        self.fp8_training = None     # quant.fp8.FP8TrainingManager: FP8 decoder linears when set
        self.cp_group = None         # context-parallel group: attention runs as a ring over it

    # -- parameter access ------------------------------------------------------
    def p(self, name: str) -> nn.Parameter:
        return self._params[name]

    def named_flat_params(self) -> Iterator[tuple[str, nn.Parameter]]:
        return iter(self._params.items())

    @property
    def lm_head(self) -> Tensor:
        return self._params["embed"] if self.args.tie_word_embeddings else self._params["lm_head"]

    def attach_main_grad(self, grad_flat: Optional[Tensor]) -> None:
        for name, p in self._params.items():
            if grad_flat is None:
                if hasattr(p, "main_grad"):
                    del p.main_grad
            else:
                p.main_grad = self.layout.view(grad_flat, name)

    @torch.no_grad()
    def init_weights(self, seed: int = 0, std: Optional[float] = None) -> None:
        """N(0, std) matrices, ones for norms; deterministic per (seed, name)
        so every rank of a sharded job builds the identical model."""
        std = self.args.init_std if std is None else std
        gen = torch.Generator(device=self.flat.device)
        for i, (name, p) in enumerate(self._params.items()):
            if is_matrix(name):
                gen.manual_seed(seed * 7919 + i)
                p.normal_(0.0, std, generator=gen)
            else:
                p.fill_(1.0)

    # -- forward ---------------------------------------------------------------
    def _linear(self, name: str, x: Tensor) -> Tensor:
        w = self._params[name]
        f8 = self.fp8_training
        if f8 is not None and f8.applies_to(name):
            return f8.linear(name, x, w)
        return ops.linear(x, w)

    def _attention_block(self, i: int, x: Tensor, positions: Tensor, cu: Tensor, max_len: int) -> Tensor:
        a = self.args
        P = self._params
        qkv = self._linear(f"layers.{i}.wqkv", x)
        qn = P.get(f"layers.{i}.q_norm")
        kn = P.get(f"layers.{i}.k_norm")
        q, k, v = ops.qk_norm_rope(qkv, qn, kn, positions, self.inv_freq, a.num_heads, a.num_kv_heads, a.head_dim,
                                   a.rms_norm_eps)
        if self.cp_group is not None:
            o = self._ring_attention(q, k, v, max_len)
        else:
            o = ops.attention_varlen(q, k, v, cu, max_len, causal=True, scale=1.0 / math.sqrt(a.head_dim))
        return self._linear(f"layers.{i}.wo", o.reshape(o.shape[0], -1))

    def _ring_attention(self, q: Tensor, k: Tensor, v: Tensor, seg: int) -> Tensor:
        """Context parallelism: the pack is B segments of ``seg`` tokens, each
        this rank's zigzag share of one sequence; attention over the whole
        sequences runs as a ring over the CP group."""
        from lumenrl_b200.parallel.context_parallel import ring_attention
        T = q.shape[0]
        B = T // seg
        to_bhtd = lambda x: x.reshape(B, seg, x.shape[1], x.shape[2]).transpose(1, 2).contiguous()  # noqa: E731
        o = ring_attention(to_bhtd(q), to_bhtd(k), to_bhtd(v), self.cp_group, 1.0 / math.sqrt(self.args.head_dim))
        return o.transpose(1, 2).reshape(T, q.shape[1], q.shape[2])

    def _mlp_block(self, i: int, h: Tensor) -> Tensor:
        P = self._params
        if self.args.is_moe_layer(i):
            from lumenrl_b200.models.moe import moe_forward
            out, aux = moe_forward(self, i, h)
            if aux is not None:
                self.aux_losses.append(aux)
            return out
        return self._linear(f"layers.{i}.w2", ops.swiglu(self._linear(f"layers.{i}.w13", h)))

    def _layer_fused(self, i: int, x: Tensor, pending: Optional[Tensor], positions: Tensor, cu: Tensor,
                     max_len: int) -> tuple[Tensor, Tensor]:
        """Decoder layer on the residual stream ``x + pending`` (``pending`` is
        the previous layer's MLP output, None for the first layer).  Returns
        (stream after attention, MLP output): the caller's next add is fused
        into the next norm, so every residual add of the stack runs inside an
        add + RMSNorm kernel (forward and backward)."""
        eps = self.args.rms_norm_eps
        P = self._params
        h, x = ops.add_rmsnorm(x, pending, P[f"layers.{i}.ln1"], eps)
        a = self._attention_block(i, h, positions, cu, max_len)
        h, x = ops.add_rmsnorm(x, a, P[f"layers.{i}.ln2"], eps)
        return x, self._mlp_block(i, h)

    def _layer(self, i: int, x: Tensor, positions: Tensor, cu: Tensor, max_len: int) -> Tensor:
        s, m = self._layer_fused(i, x, None, positions, cu, max_len)
        return s + m

    def forward_packed(self, ids: Tensor, positions: Tensor, cu_seqlens: Tensor, max_seqlen: int,
                       output_hidden_layers: Optional[list[int]] = None) -> Tensor | tuple[Tensor, list[Tensor]]:
        """ids/positions [T] packed by ``cu_seqlens`` -> final-normed hidden [T, H].

        ``output_hidden_layers`` additionally returns the residual stream after
        those layers (Eagle3 auxiliary states)."""
        self.aux_losses = []
        x = embed(ids, self._params["embed"])
        pending: Optional[Tensor] = None   # MLP output not yet added to the stream
        tapped: dict[int, Tensor] = {}
        want = set(output_hidden_layers or [])
        for i in range(self.args.num_layers):
            if (self.gradient_checkpointing or i in self.recompute_layers) and torch.is_grad_enabled():
                x, pending = _ckpt(self._layer_fused, i, x, pending, positions, cu_seqlens, max_seqlen,
                                   use_reentrant=False)
            else:
                x, pending = self._layer_fused(i, x, pending, positions, cu_seqlens, max_seqlen)
            if i in want:
                tapped[i] = x + pending
        h, _ = ops.add_rmsnorm(x, pending, self._params["norm"], self.args.rms_norm_eps)
        if output_hidden_layers is not None:
            return h, [tapped[i] for i in output_hidden_layers]   # requested order, repeats allowed
        return h

    def activation_bytes_per_token_layer(self) -> int:
        """bf16 bytes autograd keeps per token per decoder layer without
        recomputation: block inputs and norm outputs, qkv, q/k/v, attention
        output (kept twice: by attention and by the output projection),
        gate/up and the SwiGLU product."""
        a = self.args
        F = a.moe_intermediate_size * a.num_experts_per_tok if a.num_experts else a.intermediate_size
        return 2 * (4 * a.hidden_size + 2 * a.qkv_dim + 2 * a.q_dim + 3 * F)

    def logits(self, hidden: Tensor) -> Tensor:
        return hidden @ self.lm_head.t()

    # -- HF format ---------------------------------------------------------------
    def hf_state_dict(self, flat: Optional[Tensor] = None, fused_experts: bool = False) -> dict[str, Tensor]:
        """HF-named tensors (views where possible) of ``flat`` (default: own).
        MoE experts are spelled per expert (the safetensors checkpoint layout)
        or, with ``fused_experts``, as the fused ``experts.gate_up_proj``
        [E, 2F, H] / ``experts.down_proj`` [E, H, F] tensors of
        ``transformers`` >= 5 modules (the native layout itself)."""
        a = self.args
        src = self.flat if flat is None else flat
        v = lambda n: self.layout.view(src, n)  # noqa: E731
        out: dict[str, Tensor] = {"model.embed_tokens.weight": v("embed"), "model.norm.weight": v("norm")}
        if not a.tie_word_embeddings:
            out["lm_head.weight"] = v("lm_head")
        for i in range(a.num_layers):
            p, hp = f"layers.{i}.", f"model.layers.{i}."
            out[hp + "input_layernorm.weight"] = v(p + "ln1")
            out[hp + "post_attention_layernorm.weight"] = v(p + "ln2")
            qkv = v(p + "wqkv")
            out[hp + "self_attn.q_proj.weight"] = qkv[: a.q_dim]
            out[hp + "self_attn.k_proj.weight"] = qkv[a.q_dim: a.q_dim + a.kv_dim]
            out[hp + "self_attn.v_proj.weight"] = qkv[a.q_dim + a.kv_dim:]
            out[hp + "self_attn.o_proj.weight"] = v(p + "wo")
            if a.qk_norm:
                out[hp + "self_attn.q_norm.weight"] = v(p + "q_norm")
                out[hp + "self_attn.k_norm.weight"] = v(p + "k_norm")
            if a.is_moe_layer(i):
                out[hp + "mlp.gate.weight"] = v(p + "router")
                w13, w2 = v(p + "experts_w13"), v(p + "experts_w2")
                F = a.moe_intermediate_size
                if fused_experts:
                    out[hp + "mlp.experts.gate_up_proj"] = w13
                    out[hp + "mlp.experts.down_proj"] = w2
                    continue
                for e in range(a.num_experts):
                    out[hp + f"mlp.experts.{e}.gate_proj.weight"] = w13[e, :F]
                    out[hp + f"mlp.experts.{e}.up_proj.weight"] = w13[e, F:]
                    out[hp + f"mlp.experts.{e}.down_proj.weight"] = w2[e]
            else:
                w13 = v(p + "w13")
                F = a.intermediate_size
                out[hp + "mlp.gate_proj.weight"] = w13[:F]
                out[hp + "mlp.up_proj.weight"] = w13[F:]
                out[hp + "mlp.down_proj.weight"] = v(p + "w2")
        return out

    @torch.no_grad()
    def load_hf_state_dict(self, sd: dict[str, Tensor], strict: bool = True) -> list[str]:
        """Load HF-named tensors, experts in either spelling (per expert or
        fused); ``strict`` rejects a dict that leaves a parameter unloaded or
        carries a tensor matching no parameter."""
        from lumenrl_b200.sync.moe_weights import split_experts
        sd = split_experts(sd)
        targets = self.hf_state_dict()
        missing = []
        for k, dst in targets.items():
            if k in sd:
                dst.copy_(sd[k].to(dst.dtype).view(dst.shape))
            else:
                missing.append(k)
        if self.args.tie_word_embeddings and "lm_head.weight" in sd and "model.embed_tokens.weight" not in sd:
            targets["model.embed_tokens.weight"].copy_(sd["lm_head.weight"])
            missing = [m for m in missing if m != "model.embed_tokens.weight"]
        if strict:
            # sync coverage: every parameter loaded, and no tensor of the
            # state dict silently dropped (a renamed or foreign key)
            extra = [k for k in sd if k not in targets and not (k == "lm_head.weight" and self.args.tie_word_embeddings)]
            if missing or extra:
                raise KeyError(f"weight sync coverage: missing {missing[:8]}{'...' if len(missing) > 8 else ''}, "
                               f"unexpected {extra[:8]}{'...' if len(extra) > 8 else ''}")
        return missing
