"""Forward passes of the rollout engine over the paged KV cache.

* ``prefill``: packed prompts, causal varlen attention over the prompt itself,
  K/V written into the cache, logits of each prompt's last token.
* ``decode``: one token per sequence; QK-norm+RoPE, KV append and paged
  attention per layer, then the LM head.  Shapes are static, so the whole step
  is captured once per batch size into a CUDA graph (``DecodeGraph``): a
  ~36-layer step is ~400 launches that the graph replays with one.

The math is the training model's (same kernels for RMSNorm, QK-norm+RoPE,
SwiGLU), which keeps rollout and training log-probs consistent.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor

from lumenrl_b200 import ops
from lumenrl_b200.engine.inference.kv_cache import PagedKVCache
from lumenrl_b200.models.qwen3 import Qwen3Model


class TPShards:
    """Tensor-parallel rollout (Megatron layout) for one rank of a TP group:
    this rank's slice of every decoder linear, rebuilt from the full bf16
    weights at each weight sync (``refresh``).

    * ``wqkv``: the q rows of heads [t Hq/T, (t+1) Hq/T) and the k / v rows of
      kv heads [t Hk/T, (t+1) Hk/T) (column parallel: no reduction);
    * ``wo``: the matching input columns (row parallel: partial sums);
    * ``w13``: rows [t F/T, (t+1) F/T) of gate and of up (column parallel);
    * ``w2``: the matching input columns (row parallel).

    Norm weights, the embedding and the LM head stay replicated, so after the
    two all-reduces of a layer every rank holds the same residual stream and
    samples the same tokens.  The KV cache of a rank holds its kv heads only."""

    SHARDED = ("wqkv", "wo", "w13", "w2")

    def __init__(self, model: Qwen3Model, group, rank: int, size: int) -> None:
        a = model.args
        if a.num_heads % size or a.num_kv_heads % size or a.intermediate_size % size:
            raise ValueError(f"rollout TP={size} must divide heads ({a.num_heads} q / {a.num_kv_heads} kv) and "
                             f"the FFN width ({a.intermediate_size})")
        if a.num_experts:
            raise ValueError("rollout TP serves dense models; MoE rollouts shard experts instead")
        self.model, self.group, self.rank, self.size = model, group, rank, size
        self.num_heads, self.num_kv_heads = a.num_heads // size, a.num_kv_heads // size
        self.weights: dict[str, Tensor] = {}
        self.refresh()

    @torch.no_grad()
    def _slice(self, kind: str, w: Tensor) -> Tensor:
        a, t, T = self.model.args, self.rank, self.size
        D = a.head_dim
        if kind == "wqkv":
            qh, kh = self.num_heads * D, self.num_kv_heads * D
            q0, k0 = a.num_heads * D, a.num_heads * D + a.num_kv_heads * D
            return torch.cat([w[t * qh:(t + 1) * qh], w[q0 + t * kh: q0 + (t + 1) * kh],
                              w[k0 + t * kh: k0 + (t + 1) * kh]])
        if kind == "wo":
            qh = self.num_heads * D
            return w[:, t * qh:(t + 1) * qh]
        F, f = a.intermediate_size, a.intermediate_size // T
        if kind == "w13":
            return torch.cat([w[t * f:(t + 1) * f], w[F + t * f: F + (t + 1) * f]])
        return w[:, t * f:(t + 1) * f]    # w2

    @torch.no_grad()
    def refresh(self) -> None:
        """Copy this rank's slices out of the model's (full, current) weights,
        into the same buffers every time (captured decode graphs stay valid)."""
        for name, p in self.model.named_flat_params():
            kind = name.rsplit(".", 1)[-1]
            if kind not in self.SHARDED:
                continue
            sl = self._slice(kind, p.detach())
            dst = self.weights.get(name)
            if dst is None:
                self.weights[name] = sl.contiguous().clone()
            else:
                dst.copy_(sl)

    def reduce(self, x: Tensor) -> Tensor:
        """Sum the row-parallel partial outputs over the TP group (in place)."""
        import torch.distributed as dist
        dist.all_reduce(x, group=self.group)
        return x


class ModelRunner:
    def __init__(self, model: Qwen3Model, cache: PagedKVCache, tp: Optional[TPShards] = None) -> None:
        self.model = model
        self.cache = cache
        self.tp = tp
        self.args = model.args
        self.scale = 1.0 / math.sqrt(self.args.head_dim)
        self.routing_recorder = None
        self.max_len = 0   # static bound on context length (set by the engine)
        self.fp8 = None    # FP8RolloutQuantizer: W8A8 blockwise linears when set
        # token ids >= vocab_limit (the padded rows of the embedding / LM head
        # that no tokenizer id maps to) are never sampled: the LM head is
        # applied to its first vocab_limit rows only, which is the same as
        # masking the out-of-vocabulary logits to -inf before the softmax
        self.vocab_limit: Optional[int] = None

    def _lin(self, x: Tensor, name: str, decode: bool) -> Tensor:
        w = self._w(name)
        if self.fp8 is not None and name in self.fp8.weights:
            return self.fp8.linear(name, x, w, decode)
        return ops.decode_linear(x, w) if decode else ops.linear(x, w)

    def _lm_head(self) -> Tensor:
        w = self.model.lm_head.detach()
        v = self.vocab_limit
        return w if v is None or v >= w.shape[0] else w[:v]

    def _w(self, name: str) -> Tensor:
        if self.tp is not None and name in self.tp.weights:
            return self.tp.weights[name]
        return self.model.p(name).detach()

    def _heads(self) -> tuple[int, int]:
        if self.tp is not None:
            return self.tp.num_heads, self.tp.num_kv_heads
        return self.args.num_heads, self.args.num_kv_heads

    def _row_parallel(self, x: Tensor, name: str, decode: bool) -> Tensor:
        y = self._lin(x, name, decode)
        return self.tp.reduce(y) if self.tp is not None else y

    def _mlp(self, i: int, h: Tensor, decode: bool = False) -> Tensor:
        if self.args.is_moe_layer(i):
            from lumenrl_b200.models.moe import moe_forward
            prev = getattr(self.model, "routing_recorder", None)
            self.model.routing_recorder = self.routing_recorder
            try:
                out, _ = moe_forward(self.model, i, h)
            finally:
                self.model.routing_recorder = prev
            return out
        return self._row_parallel(ops.swiglu(self._lin(h, f"layers.{i}.w13", decode)), f"layers.{i}.w2", decode)

    def _qkv(self, i: int, h: Tensor, positions: Tensor, slots: Tensor, decode: bool = False):
        a, c = self.args, self.cache
        qkv = self._lin(h, f"layers.{i}.wqkv", decode)
        qn = self._w(f"layers.{i}.q_norm") if a.qk_norm else None
        kn = self._w(f"layers.{i}.k_norm") if a.qk_norm else None
        nh, nkv = self._heads()
        return ops.qk_norm_rope_cache(qkv, qn, kn, positions, self.model.inv_freq, nh, nkv,
                                      a.head_dim, a.rms_norm_eps, c.k[i], c.v[i], slots, c.k_scale[i], c.v_scale[i])

    @torch.no_grad()
    def prefill(self, ids: Tensor, positions: Tensor, cu_seqlens: Tensor, max_len: int, slots: Tensor) -> Tensor:
        a, c = self.args, self.cache
        x = torch.nn.functional.embedding(ids, self._w("embed"))
        res = None
        for i in range(a.num_layers):
            h, res = ops.add_rmsnorm(x, res, self._w(f"layers.{i}.ln1"), a.rms_norm_eps)
            q, k, v = self._qkv(i, h, positions, slots)
            o = ops.attention_varlen(q, k, v, cu_seqlens, max_len, causal=True, scale=self.scale)
            x = self._row_parallel(o.reshape(o.shape[0], -1), f"layers.{i}.wo", False)
            h, res = ops.add_rmsnorm(x, res, self._w(f"layers.{i}.ln2"), a.rms_norm_eps)
            x = self._mlp(i, h)
        last = cu_seqlens[1:] - 1
        h, _ = ops.add_rmsnorm(x[last], res[last], self._w("norm"), a.rms_norm_eps)
        return ops.linear(h, self._lm_head())

    @torch.no_grad()
    def decode(self, ids: Tensor, positions: Tensor, slots: Tensor, block_table: Tensor, seq_lens: Tensor,
               shared: Optional[tuple] = None) -> Tensor:
        """``shared = (prefix_len [B] int32, group, max_prefix, max_suffix)``:
        rows of each group of ``group`` share their first ``prefix_len``
        tokens' KV blocks, and attention reads those once per group."""
        a, c = self.args, self.cache
        x = torch.nn.functional.embedding(ids, self._w("embed"))
        res = None
        for i in range(a.num_layers):
            h, res = ops.add_rmsnorm(x, res, self._w(f"layers.{i}.ln1"), a.rms_norm_eps)
            q, k, v = self._qkv(i, h, positions, slots, True)
            if shared is not None:
                o = ops.paged_decode_attention_shared(q, c.k[i], c.v[i], block_table, seq_lens, shared[0], shared[1],
                                                      self.scale, c.k_scale[i], c.v_scale[i], shared[2], shared[3])
            else:
                o = ops.paged_decode_attention(q, c.k[i], c.v[i], block_table, seq_lens, self.scale,
                                               c.k_scale[i], c.v_scale[i], self.max_len)
            x = self._row_parallel(o.reshape(o.shape[0], -1), f"layers.{i}.wo", True)
            h, res = ops.add_rmsnorm(x, res, self._w(f"layers.{i}.ln2"), a.rms_norm_eps)
            x = self._mlp(i, h, True)
        h, _ = ops.add_rmsnorm(x, res, self._w("norm"), a.rms_norm_eps)
        return ops.decode_linear(h, self._lm_head())


class RoutingRecorder:
    """Expert ids chosen by every MoE layer in the last forward (rollout
    routing replay, R3): ``record`` keeps the layer's id tensor as int16, so
    inside a captured decode graph the recorded tensors are graph buffers
    that every replay rewrites; ``take`` stacks them into a new tensor."""

    def __init__(self, layers: list[int]) -> None:
        self.layers = layers
        self.buf: dict[int, Tensor] = {}

    def record(self, layer: int, ids: Tensor) -> None:
        self.buf[layer] = ids.to(torch.int16)

    def take(self) -> Tensor:
        return torch.stack([self.buf[l] for l in self.layers], dim=1)  # [B, layers, k]


class DecodeGraph:
    """Static-shape decode step + sampling, captured into one CUDA graph.

    Inputs live in static buffers that the caller updates in place
    (``tokens``, ``positions``, ``block_table``, ``row_seed``, ``step``,
    ``prefix_len``); ``seq_lens`` and ``slots`` are derived inside the graph.
    ``share = (group, max_prefix, max_suffix)`` selects shared-prefix
    attention with those static bounds."""

    def __init__(self, runner: ModelRunner, batch: int, max_blocks: int, temperature: float, top_p: float,
                 use_graph: bool, share: Optional[tuple] = None) -> None:
        dev = runner.cache.device
        self.runner = runner
        self.B = batch
        self.bs = runner.cache.spec.block_size
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.long, device=dev)
        self.block_table = torch.zeros(batch, max_blocks, dtype=torch.int32, device=dev)
        self.row_seed = torch.zeros(batch, dtype=torch.long, device=dev)
        self.step = torch.zeros(batch, dtype=torch.long, device=dev)   # token index per row
        self.prefix_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.share = share
        self.temperature, self.top_p = temperature, top_p
        # MoE models: this step's routes, recorded by the graph's own recorder
        # (a recorder created per generate() call would not see a cached
        # graph's replays)
        moe_layers = [i for i in range(runner.args.num_layers) if runner.args.is_moe_layer(i)]
        self.recorder = RoutingRecorder(moe_layers) if moe_layers else None
        self.out_tokens: Optional[Tensor] = None
        self.out_logp: Optional[Tensor] = None
        self.graph = None
        if use_graph and dev.type == "cuda":
            self._capture()

    def _body(self) -> None:
        pos = self.positions
        blk = self.block_table.gather(1, (pos // self.bs).unsqueeze(1).to(torch.long)).squeeze(1).to(torch.long)
        slots = blk * self.bs + pos % self.bs
        seq_lens = (pos + 1).to(torch.int32)
        shared = (self.prefix_len, *self.share) if self.share is not None else None
        prev = self.runner.routing_recorder
        self.runner.routing_recorder = self.recorder if self.recorder is not None else prev
        try:
            logits = self.runner.decode(self.tokens, pos, slots, self.block_table, seq_lens, shared)
        finally:
            self.runner.routing_recorder = prev
        tok, lp = ops.sample_tokens_device(logits, self.temperature, self.top_p, self.row_seed, self.step)
        if self.out_tokens is None:
            self.out_tokens, self.out_logp = tok, lp
        else:
            self.out_tokens.copy_(tok)
            self.out_logp.copy_(lp)

    def _capture(self) -> None:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._body()
        torch.cuda.current_stream().wait_stream(s)
        from lumenrl_b200.ops.ext import LAUNCHES
        g = torch.cuda.CUDAGraph()
        before = LAUNCHES[0]
        with torch.cuda.graph(g):
            self._body()
        self.graph = g
        self.launches_per_replay = LAUNCHES[0] - before

    def run(self) -> tuple[Tensor, Tensor]:
        if self.graph is not None:
            from lumenrl_b200.ops.ext import LAUNCHES
            self.graph.replay()
            LAUNCHES[0] += self.launches_per_replay
        else:
            self._body()
        return self.out_tokens, self.out_logp
