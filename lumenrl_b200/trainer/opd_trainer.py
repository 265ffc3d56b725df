"""On-policy distillation (reference ``lumenrl/trainer/opd_trainer.py:35-811``).

Per step: the student samples responses with the native engine; a frozen
teacher scores the same sequences; the student minimises the full-vocabulary
KL (``reverse`` = KL(student || teacher), ``forward`` = KL(teacher ||
student)) at temperature ``T`` over response tokens, optionally weighted by
``position_decay ** t``.  Multi-teacher routing: rows carry a routing key
(``distillation.teacher_key``, e.g. ``data_source``) and each key maps to its
own teacher.  Logits are never materialised for the whole batch: the student
and teacher LM heads run per chunk of tokens inside the loss.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from lumenrl_b200 import ops
from lumenrl_b200.engine.training.actor import ActorEngine
from lumenrl_b200.engine.training.packing import make_micro_batches, pack_from_grid
from lumenrl_b200.trainer.rl_trainer import RLTrainer


def chunked_vocab_kl(student_h: torch.Tensor, student_w: torch.Tensor, teacher_h: torch.Tensor,
                     teacher_w: torch.Tensor, direction: str, temperature: float, weights: torch.Tensor,
                     chunk: int = 1024) -> torch.Tensor:
    """sum_t weights[t] * KL_t over the full vocabulary, chunked over tokens."""
    total = student_h.new_zeros((), dtype=torch.float32)
    for a in range(0, student_h.shape[0], chunk):
        b = min(student_h.shape[0], a + chunk)
        ls = F.log_softmax((student_h[a:b] @ student_w.t()).float() / temperature, -1)
        with torch.no_grad():
            lt = F.log_softmax((teacher_h[a:b] @ teacher_w.t()).float() / temperature, -1)
        if direction == "reverse":
            kl = (ls.exp() * (ls - lt)).sum(-1)
        else:
            kl = (lt.exp() * (lt - ls)).sum(-1)
        total = total + (kl * weights[a:b]).sum()
    return total


class OPDTrainer(RLTrainer):
    def setup(self) -> "OPDTrainer":
        super().setup()
        self.teachers: dict[str, ActorEngine] = {}
        default = ActorEngine(self.model_args, self.state, seed=self.config.seed + 1, trainable=False)
        self.teachers["default"] = default
        return self

    def add_teacher(self, key: str, engine: ActorEngine) -> None:
        self.teachers[key] = engine

    def step(self) -> dict:
        c, st = self.config, self.state
        oc = c.algorithm.opd
        batch = self._rollout(self.global_step)
        t = batch.tensors
        mask = t["response_mask"].float()
        total_tok = max(float(mask.sum()), 1.0)
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        keys = batch.meta.get(c.algorithm.distillation.teacher_key) or ["default"] * len(batch)
        kl_sum = 0.0
        for rows in make_micro_batches(lens, rows_per_micro=self.spec.rows_per_micro):
            pb = pack_from_grid(t["prompt_ids"], t["prompt_lengths"], t["responses"], t["response_lengths"], rows,
                                st.device)
            sm = self.actor.model
            hs = sm.forward_packed(pb.input_ids, pb.positions, pb.cu_seqlens, pb.max_seqlen).index_select(
                0, pb.score_index)
            r_idx = torch.as_tensor(rows, device=st.device)[pb.out_row]
            w = mask[r_idx, pb.out_col]
            if oc.position_weighting:
                w = w * (oc.position_decay ** pb.out_col.float())
            teacher = self.teachers.get(keys[rows[0]], self.teachers["default"])
            with torch.no_grad():
                ht = teacher.model.forward_packed(pb.input_ids, pb.positions, pb.cu_seqlens, pb.max_seqlen
                                                  ).index_select(0, pb.score_index)
            loss = chunked_vocab_kl(hs, sm.lm_head, ht, teacher.model.lm_head.detach(), oc.kl_direction,
                                    oc.temperature, w) * oc.opd_coeff / total_tok
            loss.backward()
            kl_sum += float(loss.detach())
        opt = self.actor.opt.step(self.actor.sched.current if self.actor.sched else None)
        self.rollout.update_weights()
        self.global_step += 1
        m = {"opd/kl": kl_sum, "actor/grad_norm": opt["grad_norm"], "step": self.global_step}
        self.history.append(m)
        return m
