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

    def step(self, ids: Optional[torch.Tensor] = None) -> dict:
        st, sp = self.state, self.spec
        dev = st.device
        t0 = time.perf_counter()
        if ids is None:
            g = torch.Generator().manual_seed(self.seed * 1_000_003 + self.step_count * 7919 + st.rank)
            ids = torch.randint(0, self.args.vocab_size, (sp.batch_per_rank * sp.seq_len,), generator=g).to(dev)
        cu = torch.arange(0, ids.numel() + 1, sp.seq_len, dtype=torch.int32, device=dev)
        aux, last = self.teacher_forward(ids, cu)
        if sp.draft_type == "dflash":
            B = ids.numel() // sp.seq_len
            K = sp.num_target_layers
            feats = last if K == 1 else aux[:, -K * self.args.hidden_size:]
            out = self.draft(feats.view(B, sp.seq_len, -1), self.teacher.lm_head, target_ids=ids.view(B, sp.seq_len),
                             loss_decay_gamma=sp.loss_decay_gamma, return_logits=False)
            acc = [float(out["accuracy"])]
        else:
            out = self.draft(ids, aux, last, self.teacher.p("embed").detach(), self.teacher.lm_head.detach(), cu,
                             torch.ones_like(ids, dtype=torch.float32), decay=sp.position_decay)
            acc = [float(a) for a in out["accuracies"]]
        out["loss"].backward()
        if dist.is_initialized() and st.world_size > 1:
            allreduce_mean_grads(list(self.draft.parameters()), st.world_size)
        o = self.opt.step()
        self.step_count += 1
        return {"loss": float(out["loss"].detach()), "grad_norm": o["grad_norm"],
                "acc": acc, "step_s": time.perf_counter() - t0,
                "tokens": int(ids.numel()) * st.world_size}


def allreduce_mean_grads(params: list, world: int, bucket_bytes: int = 256 << 20) -> None:
    """Replicated data parallel: average gradients across ranks with a few
    large flat all-reduces (one per dtype bucket) instead of one per tensor."""
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
            dist.all_reduce(flat)
            flat /= world
            off = 0
            for g in gs[i:j]:
                g.copy_(flat[off: off + g.numel()].view_as(g))
                off += g.numel()
            i = j
