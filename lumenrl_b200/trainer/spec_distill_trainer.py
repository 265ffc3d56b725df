"""Speculative-decoding draft distillation (Eagle3 or DFlash draft; SDDD).

Reference: ``lumenrl/trainer/spec_distill_trainer.py:41-2286``.  There the
teacher runs in an inference engine on rank 0 and ships hidden states through
Mooncake/MORI RDMA and /dev/shm slot files.  Here:

* teacher ranks run the frozen teacher's packed forward and tap the auxiliary
  layers (e.g. 2, 18, 33) and the final-normed hidden state;
* draft ranks train the Eagle3 head (TTT unroll, forward KL over the draft
  vocabulary, ``position_decay ** step`` weights) with the bf16/fp32-master
  optimizer, gradients all-reduced across draft ranks (replicated data
  parallel);
* teacher -> draft hidden states move over NVLink through
  ``transfer.p2p_ring.HiddenStateRing`` (teacher pushes rows into the draft
  GPU's ring slot, bounded-wait ready flags); in a single process the
  teacher and draft share the GPU and the hand-off is a tensor.

``SpecDistillTrainer.step()`` consumes one global batch of ``seq_len``-token
sequences and returns loss/accuracy per TTT step (Eagle3) or the
decay-weighted CE and accuracy (DFlash, ``draft_type="dflash"``: fed the
final hidden state, or the last ``num_target_layers`` aux taps).
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from lumenrl_b200.models.config import ModelArgs
from lumenrl_b200.models.dflash import DFlashModel
from lumenrl_b200.models.eagle3 import Eagle3Model
from lumenrl_b200.models.qwen3 import Qwen3Model
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.bf16_optimizer import BF16Optimizer


@dataclass
class SpecDistillSpec:
    aux_layers: tuple = (2, 18, 33)
    draft_vocab: int = 32000
    ttt_length: int = 7
    position_decay: float = 0.8
    seq_len: int = 2048
    batch_per_rank: int = 8
    lr: float = 1e-4
    draft_heads: int = 32
    draft_kv_heads: int = 8
    draft_ffn: Optional[int] = None
    draft_type: str = "eagle3"          # or "dflash"
    draft_layers: int = 2               # DFlash blocks
    num_target_layers: int = 1          # DFlash: teacher layers fused
    loss_decay_gamma: float = 7.0       # DFlash CE position decay


class SpecDistillTrainer:
    def __init__(self, teacher_args: ModelArgs, spec: SpecDistillSpec, state: ParallelState, seed: int = 0,
                 total_steps: int = 1000) -> None:
        self.args, self.spec, self.state = teacher_args, spec, state
        dev = state.device
        dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        self.teacher = Qwen3Model(teacher_args, device=dev, dtype=dtype, requires_grad=False)
        self.teacher.init_weights(seed)
        a = teacher_args
        if spec.draft_type == "dflash":
            if spec.num_target_layers > max(1, len(spec.aux_layers)):
                raise ValueError("num_target_layers exceeds the tapped teacher layers")
            torch.manual_seed(seed)
            self.draft = DFlashModel(a.hidden_size, spec.num_target_layers, max(1, a.hidden_size // 128),
                                     spec.draft_layers, block_size=8).to(device=dev, dtype=dtype)
        elif spec.draft_type == "eagle3":
            self.draft = Eagle3Model(a.hidden_size, a.vocab_size, spec.draft_vocab, spec.draft_heads,
                                     spec.draft_kv_heads, a.head_dim, spec.draft_ffn or a.intermediate_size, 1,
                                     spec.ttt_length, a.rms_norm_eps, a.rope_theta,
                                     vocab_seed=seed).to(device=dev, dtype=dtype)
        else:
            raise ValueError(f"unknown draft_type {spec.draft_type!r} (eagle3 or dflash)")
        self.opt = BF16Optimizer(self.draft.parameters(), lr=spec.lr, total_steps=total_steps)
        self.seed = seed
        self.step_count = 0

    @torch.no_grad()
    def teacher_forward(self, ids: torch.Tensor, cu: torch.Tensor):
        lens = (cu[1:] - cu[:-1]).tolist()
        pos = torch.cat([torch.arange(n, device=ids.device) for n in lens])
        h, taps = self.teacher.forward_packed(ids, pos, cu, max(lens), output_hidden_layers=list(self.spec.aux_layers))
        return torch.cat(taps, -1), h

    def _ids(self, step: int, source: int) -> torch.Tensor:
        """Synthetic batch of ``batch_per_rank`` sequences for (step, source
        rank): uniform token ids, identical on every process that asks."""
        sp = self.spec
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + step * 7919 + source)
        return torch.randint(0, self.args.vocab_size, (sp.batch_per_rank * sp.seq_len,), generator=g)

    def draft_loss(self, ids: torch.Tensor, aux: torch.Tensor, last: torch.Tensor) -> tuple:
        sp = self.spec
        dev = ids.device
        cu = torch.arange(0, ids.numel() + 1, sp.seq_len, dtype=torch.int32, device=dev)
        if sp.draft_type == "dflash":
            B = ids.numel() // sp.seq_len
            K = sp.num_target_layers
            feats = last if K == 1 else aux[:, -K * self.args.hidden_size:]
            out = self.draft(feats.view(B, sp.seq_len, -1), self.lm_head_weight(), target_ids=ids.view(B, sp.seq_len),
                             loss_decay_gamma=sp.loss_decay_gamma, return_logits=False)
            return out["loss"], [float(out["accuracy"])]
        out = self.draft(ids, aux, last, self.embed_weight(), self.lm_head_weight(), cu,
                         torch.ones_like(ids, dtype=torch.float32), decay=sp.position_decay)
        return out["loss"], [float(a) for a in out["accuracies"]]

    def embed_weight(self) -> torch.Tensor:
        return self.teacher.p("embed").detach()

    def lm_head_weight(self) -> torch.Tensor:
        return self.teacher.lm_head.detach()

    def draft_update(self, batches: list, group=None, world: int = 1, comm=None) -> dict:
        """One optimizer step of the draft over ``batches`` = [(ids, aux,
        last), ...]: the loss is the mean over batches (gradients accumulate),
        then gradients are averaged over ``world`` draft replicas."""
        accs: list = []
        total = 0.0
        for ids, aux, last in batches:
            loss, acc = self.draft_loss(ids, aux, last)
            (loss / len(batches)).backward()
            total += float(loss.detach()) / len(batches)
            accs.append(acc)
        if world > 1:
            allreduce_mean_grads(list(self.draft.parameters()), world, group=group, comm=comm)
        o = self.opt.step()
        self.step_count += 1
        mean_acc = [sum(a[i] for a in accs) / len(accs) for i in range(len(accs[0]))]
        return {"loss": total, "grad_norm": o["grad_norm"], "acc": mean_acc}

    def step(self, ids: Optional[torch.Tensor] = None) -> dict:
        st, sp = self.state, self.spec
        dev = st.device
        t0 = time.perf_counter()
        if ids is None:
            ids = self._ids(self.step_count, st.rank).to(dev)
        cu = torch.arange(0, ids.numel() + 1, sp.seq_len, dtype=torch.int32, device=dev)
        aux, last = self.teacher_forward(ids, cu)
        world = st.world_size if (dist.is_initialized() and st.world_size > 1) else 1
        out = self.draft_update([(ids, aux, last)], world=world)
        out.update(step_s=time.perf_counter() - t0, tokens=int(ids.numel()) * st.world_size)
        return out


class SDDDTrainer(SpecDistillTrainer):
    """Teacher / draft split over GPUs (reference layout: teacher on its own
    ranks with shared-memory ring slots and a hidden-state broadcast,
    ``lumenrl/trainer/spec_distill_trainer.py:94-283, 943-963``; train loop
    ``:1894-2243``).

    Ranks ``[0, num_teacher)`` run the frozen teacher's packed forward; ranks
    ``[num_teacher, world)`` train the draft.  Teacher rank ``t`` streams
    each batch -- its token ids plus the tapped auxiliary layers and the
    final-normed hidden state -- to draft rank ``num_teacher + t % num_draft``
    through a ``HiddenStateRing`` (peer stores into the draft GPU's slot over
    NVLink, bounded-wait flags; send/recv over the process group on CPU).
    Each draft step consumes one batch from every teacher feeding it,
    accumulates gradients over them, averages gradients over the draft
    replicas and steps the optimizer.  With ``nslots`` ring slots a teacher
    runs up to ``nslots`` batches ahead of its draft, so teacher forwards
    overlap draft training.  The draft ranks hold copies of the teacher's
    embedding, final LM head (broadcast from teacher rank 0 at start-up); the
    teacher decoder stays on the teacher ranks."""

    def __init__(self, teacher_args: ModelArgs, spec: SpecDistillSpec, state: ParallelState, num_teacher: int,
                 seed: int = 0, total_steps: int = 1000, nslots: int = 2) -> None:
        from lumenrl_b200.transfer.p2p_ring import HiddenStateRing
        world, rank = state.world_size, state.rank
        if not 0 < num_teacher < world:
            raise ValueError(f"num_teacher={num_teacher} must leave at least one draft rank of {world}")
        self.num_teacher, self.num_draft = num_teacher, world - num_teacher
        self.is_teacher = rank < num_teacher
        self.args, self.spec, self.state, self.seed, self.step_count = teacher_args, spec, state, seed, 0
        dev = state.device
        dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        self.dtype = dtype
        a = teacher_args
        self.feat_dim = (len(spec.aux_layers) + 1) * a.hidden_size
        T = spec.batch_per_rank * spec.seq_len
        self.payload_bytes = T * self.feat_dim * torch.empty(0, dtype=dtype).element_size() + T * 4
        # every rank creates every group in the same order (collective)
        self.pair_groups = [dist.new_group([t, self.consumer_of(t)]) for t in range(num_teacher)]
        self.draft_group = dist.new_group(list(range(num_teacher, world)))
        self.weights_group = dist.new_group([0] + list(range(num_teacher, world)))
        if self.is_teacher:
            self.teacher = Qwen3Model(a, device=dev, dtype=dtype, requires_grad=False)
            self.teacher.init_weights(seed)
            self.draft, self.opt = None, None
            self._embed = self.teacher.p("embed").detach()
            self._lm_head = self.teacher.lm_head.detach()
        else:
            self.teacher = None
            self._embed = torch.empty(a.vocab_size, a.hidden_size, dtype=dtype, device=dev)
            self._lm_head = self._embed if a.tie_word_embeddings else torch.empty(a.vocab_size, a.hidden_size,
                                                                                 dtype=dtype, device=dev)
            self._build_draft(dev, dtype, total_steps)
        # the draft replicas average gradients with the NVLink all-reduce kernel
        # (LRL_DRAFT_ALLREDUCE=nccl keeps NCCL); every draft rank builds it
        self.ar_comm = None
        if (not self.is_teacher and self.num_draft > 1 and dev.type == "cuda"
                and os.environ.get("LRL_DRAFT_ALLREDUCE", "nvlink") != "nccl"):
            from lumenrl_b200.parallel.symm import NVLinkAllReduce
            n_grad = sum(p.numel() for p in self.draft.parameters())
            self.ar_comm = NVLinkAllReduce(min(n_grad, 64 << 20), rank - num_teacher, self.num_draft,
                                           group=self.draft_group)
        if rank in [0] + list(range(num_teacher, world)):
            dist.broadcast(self._embed, src=0, group=self.weights_group)
            if not a.tie_word_embeddings:
                dist.broadcast(self._lm_head, src=0, group=self.weights_group)
        self.rings: dict[int, "HiddenStateRing"] = {}
        for t in range(num_teacher):
            d = self.consumer_of(t)
            if rank in (t, d):
                # ring ranks are group-local: the teacher is 0, the draft 1
                self.rings[t] = HiddenStateRing(0, 1, self.payload_bytes, nslots, group=self.pair_groups[t])
        self.producers = [t for t in range(num_teacher) if self.consumer_of(t) == rank]

    def consumer_of(self, teacher_rank: int) -> int:
        return self.num_teacher + teacher_rank % self.num_draft

    def _build_draft(self, dev, dtype, total_steps: int) -> None:
        sp, a = self.spec, self.args
        torch.manual_seed(self.seed)
        if sp.draft_type == "dflash":
            self.draft = DFlashModel(a.hidden_size, sp.num_target_layers, max(1, a.hidden_size // 128),
                                     sp.draft_layers, block_size=8).to(device=dev, dtype=dtype)
        else:
            self.draft = Eagle3Model(a.hidden_size, a.vocab_size, sp.draft_vocab, sp.draft_heads, sp.draft_kv_heads,
                                     a.head_dim, sp.draft_ffn or a.intermediate_size, 1, sp.ttt_length,
                                     a.rms_norm_eps, a.rope_theta, vocab_seed=self.seed).to(device=dev, dtype=dtype)
        self.opt = BF16Optimizer(self.draft.parameters(), lr=sp.lr, total_steps=total_steps)

    def embed_weight(self) -> torch.Tensor:
        return self._embed

    def lm_head_weight(self) -> torch.Tensor:
        return self._lm_head

    def _pack(self, ids: torch.Tensor, aux: torch.Tensor, last: torch.Tensor) -> torch.Tensor:
        feats = torch.cat([aux, last], -1).contiguous()
        return torch.cat([feats.view(-1).view(torch.uint8), ids.to(torch.int32).view(torch.uint8)])

    def _unpack(self, payload: torch.Tensor) -> tuple:
        sp, H = self.spec, self.args.hidden_size
        T = sp.batch_per_rank * sp.seq_len
        fb = T * self.feat_dim * torch.empty(0, dtype=self.dtype).element_size()
        feats = payload[:fb].view(self.dtype).view(T, self.feat_dim)
        ids = payload[fb: fb + T * 4].view(torch.int32).to(torch.long)
        return ids, feats[:, : self.feat_dim - H], feats[:, self.feat_dim - H:]

    def step(self) -> dict:
        st, sp = self.state, self.spec
        dev = st.device
        t0 = time.perf_counter()
        tokens = sp.batch_per_rank * sp.seq_len * self.num_teacher   # draft tokens consumed per step, job-wide
        if self.is_teacher:
            ids = self._ids(self.step_count, st.rank).to(dev)
            cu = torch.arange(0, ids.numel() + 1, sp.seq_len, dtype=torch.int32, device=dev)
            aux, last = self.teacher_forward(ids, cu)
            self.rings[st.rank].put(self._pack(ids, aux, last))
            self.step_count += 1
            return {"role": "teacher", "step_s": time.perf_counter() - t0, "tokens": tokens}
        batches, held = [], []
        for t in self.producers:
            payload = self.rings[t].get((self.payload_bytes,), torch.uint8, device=dev)
            batches.append(self._unpack(payload))
            held.append(t)
        out = self.draft_update(batches, group=self.draft_group, world=self.num_draft, comm=self.ar_comm)
        if self.ar_comm is not None:
            self.ar_comm.check()
        for t in held:
            self.rings[t].release()
        out.update(role="draft", step_s=time.perf_counter() - t0, tokens=tokens)
        return out

    def check(self) -> None:
        for r in self.rings.values():
            r.check()

    def close(self) -> None:
        for r in self.rings.values():
            r.close()
        if self.ar_comm is not None:
            self.ar_comm.close()
            self.ar_comm = None


def allreduce_mean_grads(params: list, world: int, bucket_bytes: int = 256 << 20, group=None, comm=None) -> None:
    """Replicated data parallel: average gradients across ranks with a few
    large flat all-reduces (one per dtype bucket) instead of one per tensor.
    ``comm``: an ``NVLinkAllReduce`` (this package's peer-memory kernel, fp32
    sums); without it the buckets go through NCCL."""
    grads = [p.grad for p in params if p.grad is not None]
    by_dtype: dict = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    for gs in by_dtype.values():
        i = 0
        while i < len(gs):
            j, size = i, 0
            while j < len(gs) and (size == 0 or size + gs[j].numel() * gs[j].element_size() <= bucket_bytes):
                size += gs[j].numel() * gs[j].element_size()
                j += 1
            flat = torch.cat([g.reshape(-1) for g in gs[i:j]])
            if comm is not None and flat.is_cuda:
                comm.all_reduce_(flat, scale=1.0 / world)
            else:
                dist.all_reduce(flat, group=group)
                flat /= world
            off = 0
            for g in gs[i:j]:
                g.copy_(flat[off: off + g.numel()].view_as(g))
                off += g.numel()
            i = j
