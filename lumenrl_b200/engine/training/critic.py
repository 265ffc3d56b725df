"""Value model engine for PPO/GAE (reference ``lumenrl/workers/critic_worker.py:18-202``).

Backbone: the policy architecture in its own flat buffer (sharded AdamW like
the actor); head: an fp32 ``H -> 1`` projection read at the same positions
that score response tokens.  ``update`` minimises the clipped value loss
``max((V - R)^2, (clip(V, V_old +- eps) - R)^2)`` (token mean).
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from lumenrl_b200.algorithms.losses import value_loss
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.engine.training.actor import ActorEngine
from lumenrl_b200.engine.training.packing import make_micro_batches, pack_from_grid


class CriticEngine(ActorEngine):
    def __init__(self, args, state, **kw) -> None:
        kw.setdefault("fused_comm", False)
        super().__init__(args, state, **kw)
        H = args.hidden_size
        self.head = torch.nn.Linear(H, 1, device=self.device, dtype=torch.float32)
        torch.nn.init.zeros_(self.head.weight)
        torch.nn.init.zeros_(self.head.bias)
        self.head_opt = torch.optim.AdamW(self.head.parameters(), lr=kw.get("lr", 1e-5))

    def _values(self, pb) -> Tensor:
        h = self.model.forward_packed(pb.input_ids, pb.positions, pb.cu_seqlens, pb.max_seqlen)
        return self.head(h.index_select(0, pb.score_index).float()).squeeze(-1)

    @torch.no_grad()
    def compute_values(self, batch: DataProto, token_budget: int = 16384) -> Tensor:
        t = batch.tensors
        B, R = t["responses"].shape
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        out = torch.zeros(B, R, device=self.device)
        for rows in make_micro_batches(lens, token_budget=token_budget):
            pb = pack_from_grid(t["prompt_ids"], t["prompt_lengths"], t["responses"], t["response_lengths"], rows,
                                self.device)
            out[torch.as_tensor(rows, device=self.device)[pb.out_row], pb.out_col] = self._values(pb)
        return out

    def update(self, batch: DataProto, clip: float = 0.2, rows_per_micro: int = 4) -> dict:
        t = batch.tensors
        B = t["responses"].shape[0]
        mask = t["response_mask"].float()
        total = max(float(mask.sum()), 1.0)
        lens = (t["prompt_lengths"] + t["response_lengths"]).tolist()
        vl_sum = 0.0
        for rows in make_micro_batches(lens, rows_per_micro=rows_per_micro):
            pb = pack_from_grid(t["prompt_ids"], t["prompt_lengths"], t["responses"], t["response_lengths"], rows,
                                self.device)
            r = torch.as_tensor(rows, device=self.device)[pb.out_row]
            v = self._values(pb)
            old, ret, m = t["values"][r, pb.out_col], t["returns"][r, pb.out_col], mask[r, pb.out_col]
            loss = value_loss(v, old, ret, clip, mask=m) * (float(m.sum()) / total)
            loss.backward()
            vl_sum += float(loss.detach())
        st = self.opt.step(self.sched.current if self.sched else None)
        self.head_opt.step()
        self.head_opt.zero_grad(set_to_none=True)
        return {"critic/vf_loss": vl_sum, "critic/grad_norm": st["grad_norm"]}
