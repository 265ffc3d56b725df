"""Megatron-style training engine: tensor (+ sequence) x pipeline x data
parallelism over the Qwen3 dense decoder (reference
``engine/training/megatron_engine.py`` and ``megatron_native_engine.py``:
``mpu.initialize_model_parallel`` :235-242, TP/SP linears :322-341, PP via
the 1F1B schedule :1010-1085 / :1477-1636, DP gradient reduction).

Rank layout (TP fastest): ``rank = dp * (pp * tp) + stage * tp + t``.

* every rank builds the same full model (same seed), keeps the decoder
  layers of its pipeline stage as ``TPDecoderLayer`` shards (heads and MLP
  columns split over its TP group, activations sharded by sequence), plus the
  embedding on the first stage and the final norm / LM head on the last;
* ``step(micro_batches)`` runs 1F1B over the pipeline (``parallel.pipeline``),
  each stage's forward being the TP layers on its sequence shard; the last
  stage's loss is the summed token NLL of its shard's tokens;
* gradients: norm weights, embedding and LM head are replicated inside a TP
  group and see only that rank's tokens, so they are all-reduced over TP;
  then every parameter is averaged over DP; tied embeddings are summed over
  the two pipeline ends.  The optimizer is ``BF16Optimizer`` (fp32 master).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from lumenrl_b200 import ops
from lumenrl_b200.models.qwen3 import Qwen3Model, embed
from lumenrl_b200.parallel.pipeline import MicroBatch, OneFOneB, split_layers
from lumenrl_b200.parallel.tensor_parallel import TPComm, TPDecoderLayer


def make_groups(tp: int, pp: int) -> dict:
    """Create TP, PP and DP groups (every rank calls this, same order)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % (tp * pp):
        raise ValueError(f"world {world} is not a multiple of tp*pp = {tp * pp}")
    dp = world // (tp * pp)
    out = {"tp": None, "pp": None, "dp": None, "ends": None, "tp_size": tp, "pp_size": pp, "dp_size": dp}
    for d in range(dp):
        for s in range(pp):
            ranks = [d * pp * tp + s * tp + t for t in range(tp)]
            g = dist.new_group(ranks)
            if rank in ranks:
                out["tp"], out["tp_ranks"] = g, ranks
    for d in range(dp):
        for t in range(tp):
            ranks = [d * pp * tp + s * tp + t for s in range(pp)]
            g = dist.new_group(ranks)
            e = dist.new_group([ranks[0], ranks[-1]]) if pp > 1 else None
            if rank in ranks:
                out["pp"], out["pp_ranks"], out["ends"] = g, ranks, e
    for s in range(pp):
        for t in range(tp):
            ranks = [d * pp * tp + s * tp + t for d in range(dp)]
            g = dist.new_group(ranks)
            if rank in ranks:
                out["dp"], out["dp_ranks"] = g, ranks
    out["t"] = rank % tp
    out["stage"] = (rank // tp) % pp
    out["d"] = rank // (tp * pp)
    return out


class _Stage:
    """Pipeline stage whose layers are tensor-parallel with SP activations."""

    def __init__(self, engine: "MegatronEngine") -> None:
        e = self.e = engine
        self.stage, self.stages, self.group = e.g["stage"], e.g["pp_size"], e.g["pp"]
        self.first, self.last = self.stage == 0, self.stage == self.stages - 1
        self.hidden = e.args.hidden_size

    def _local(self, x: Tensor) -> Tensor:
        tp, t = self.e.g["tp_size"], self.e.g["t"]
        n = x.shape[0] // tp
        return x[t * n:(t + 1) * n]

    def forward(self, mb: MicroBatch, x: Optional[Tensor]) -> Tensor:
        e = self.e
        if self.first:
            x = self._local(embed(mb.ids, e.embed))
        for layer in e.layers:
            x = layer(x, mb.positions, mb.cu, mb.max_len)
        return x

    def loss(self, mb: MicroBatch, x: Tensor) -> Tensor:
        e = self.e
        h = ops.rmsnorm(x, e.norm, e.args.rms_norm_eps)
        if e.vocab_parallel:
            # vocabulary-parallel LM head: every TP rank scores all tokens of the
            # micro-batch against its slice of the vocabulary; the value returned
            # is this rank's token share (so the TP sum is the loss) while the
            # gradient is that of the full loss, which every rank needs for the
            # vocabulary-parallel backward
            from lumenrl_b200.parallel.vocab_parallel import vocab_parallel_token_logprob
            hf = _GatherTokens.apply(h, e.tpc)
            logp, _ = vocab_parallel_token_logprob(hf, e.lm_head, mb.targets, e.vocab_start, group=e.g["tp"])
            full = -(logp * mb.weights).sum()
            local = -(self._local(logp) * self._local(mb.weights)).sum()
            return local.detach() + (full - full.detach())
        logp, _ = ops.token_logprob(h, e.lm_head, self._local(mb.targets), want_entropy=False)
        return -(logp * self._local(mb.weights)).sum()


class _GatherTokens(torch.autograd.Function):
    """All-gather of the sequence-parallel token shards; the backward takes
    this rank's rows of a gradient that is already the same on every rank
    (the vocabulary-parallel backward sums it over the group)."""

    @staticmethod
    def forward(ctx, x, tpc):
        ctx.tpc = tpc
        return tpc.all_gather(x) if tpc.world > 1 else x

    @staticmethod
    def backward(ctx, dy):
        tpc = ctx.tpc
        n = dy.shape[0] // tpc.world
        return dy[tpc.rank * n:(tpc.rank + 1) * n].contiguous(), None


class MegatronEngine:
    def __init__(self, args, tp: int = 1, pp: int = 1, device: Optional[torch.device] = None,
                 dtype: torch.dtype = torch.float32, seed: int = 0, lr: float = 1e-4, fused: Optional[bool] = None,
                 groups: Optional[dict] = None, vocab_parallel: bool = False) -> None:
        """``vocab_parallel``: the LM head is split by rows over the TP group
        (Megatron's vocabulary-parallel output layer; untied embeddings) and
        the token log-probs come from ``parallel.vocab_parallel``."""
        if args.num_experts:
            raise ValueError("MegatronEngine covers dense decoders; MoE layers use parallel.expert_parallel")
        self.args = args
        self.device = device or torch.device("cpu")
        self.g = groups or make_groups(tp, pp)
        full = Qwen3Model(args, device=self.device, dtype=dtype, requires_grad=False)
        full.init_weights(seed)
        self.full_inv_freq = full.inv_freq
        lo, hi = split_layers(args.num_layers, self.g["pp_size"])[self.g["stage"]]
        self.layer_range = (lo, hi)
        self.tpc = TPComm(self.g["tp"], fused=fused)
        self.layers = torch.nn.ModuleList()
        for i in range(lo, hi):
            p = {k.split(".", 2)[2]: v for k, v in full.named_flat_params() if k.startswith(f"layers.{i}.")}
            self.layers.append(TPDecoderLayer(args, p, self.tpc, full.inv_freq))

        def P(t):
            return torch.nn.Parameter(t.detach().clone())
        first, last = self.g["stage"] == 0, self.g["stage"] == self.g["pp_size"] - 1
        self.embed = P(full.p("embed")) if first or (last and args.tie_word_embeddings) else None
        self.norm = P(full.p("norm")) if self.g["stage"] == self.g["pp_size"] - 1 else None
        self.vocab_parallel = bool(vocab_parallel) and self.g["tp_size"] > 1
        self.vocab_start = 0
        if self.vocab_parallel and args.tie_word_embeddings:
            raise ValueError("vocab_parallel needs untied embeddings (the embedding is not split by vocabulary)")
        if self.g["stage"] == self.g["pp_size"] - 1:
            if self.vocab_parallel:
                from lumenrl_b200.parallel.vocab_parallel import vocab_slice
                a, b = vocab_slice(args.vocab_size, self.g["t"], self.g["tp_size"])
                self.vocab_start = a
                self.lm_head = P(full.lm_head[a:b])
            else:
                self.lm_head = self.embed if args.tie_word_embeddings else P(full.lm_head)
        else:
            self.lm_head = None
        del full
        from lumenrl_b200.trainer.bf16_optimizer import BF16Optimizer
        # no clipping here: a global norm would need a reduction over the model-parallel shards
        self.opt = BF16Optimizer(self.parameters(), lr=lr, total_steps=1000, warmup_steps=0, max_grad_norm=0.0)
        self.sched = OneFOneB(_Stage(self), self.device, dtype)

    def parameters(self) -> list:
        ps = [p for layer in self.layers for p in layer.parameters()]
        for p in (self.embed, self.norm, self.lm_head):
            if p is not None and all(p is not q for q in ps):
                ps.append(p)
        return ps

    def _replicated_in_tp(self) -> list:
        ps = []
        for layer in self.layers:
            ps += [layer.ln1, layer.ln2] + [p for p in (layer.q_norm, layer.k_norm) if p is not None]
        for p in (self.embed, self.norm, None if self.vocab_parallel else self.lm_head):
            if p is not None and all(p is not q for q in ps):
                ps.append(p)
        return ps

    def sync_grads(self) -> None:
        g = self.g
        if g["tp_size"] > 1:
            for p in self._replicated_in_tp():
                if p.grad is not None:
                    dist.all_reduce(p.grad, group=g["tp"])
        ends = g["stage"] in (0, g["pp_size"] - 1)
        if g["pp_size"] > 1 and self.args.tie_word_embeddings and self.embed is not None and ends:
            if self.embed.grad is None:
                self.embed.grad = torch.zeros_like(self.embed)
            dist.all_reduce(self.embed.grad, group=g["ends"])
        if g["dp_size"] > 1:
            for p in self.parameters():
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
                dist.all_reduce(p.grad, group=g["dp"])
                p.grad /= g["dp_size"]

    def forward_backward(self, micro_batches: list, loss_scale: float = 1.0) -> float:
        """1F1B over the pipeline; returns the summed loss (all ranks, the
        pipeline's last stage summed over its TP group)."""
        total = self.sched.run(micro_batches, loss_scale)
        g = self.g
        t = torch.tensor([total], device=self.device, dtype=torch.float64)
        if g["stage"] == g["pp_size"] - 1 and g["tp_size"] > 1:
            dist.all_reduce(t, group=g["tp"])
        if g["pp_size"] > 1:   # last stage -> everyone in the pipeline
            dist.broadcast(t, src=g["pp_ranks"][-1], group=g["pp"])
        return float(t)

    def step(self, micro_batches: list, loss_scale: float = 1.0) -> dict:
        for p in self.parameters():
            p.grad = None
        loss = self.forward_backward(micro_batches, loss_scale)
        self.sync_grads()
        o = self.opt.step()
        return {"loss": loss, "grad_norm": o.get("grad_norm", 0.0)}
