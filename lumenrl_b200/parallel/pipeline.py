"""Pipeline parallelism: a 1F1B schedule over point-to-point sends
(reference: Megatron ``get_forward_backward_func`` driven from
``engine/training/megatron_engine.py:1010-1085, 1477-1636`` and
``megatron_native_engine.py:1474, 1630``, variable sequence lengths
:298-299).

Stage ``s`` of ``P`` owns a contiguous range of decoder layers; the first
stage also embeds the tokens, the last applies the final norm and the loss.
Micro-batches are packed variable-length token sets, so every activation
send is preceded by a 1-element shape message.  Sends and receives are
``torch.distributed`` point-to-point operations (NCCL on GPUs, gloo on CPU),
posted with ``batch_isend_irecv`` so a forward send and the next receive
overlap.

The schedule per stage: ``P - s - 1`` warm-up forwards, then alternate one
forward / one backward, then the remaining backwards.  Each stage keeps at
most ``P - s`` micro-batches of activations alive.  Gradients accumulate in
the parameters (``main_grad`` or ``.grad``), so an optimizer step after
``run`` sees the sum over micro-batches.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor


def split_layers(num_layers: int, stages: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) layer ranges, sizes differing by at most one."""
    base, extra = divmod(num_layers, stages)
    out, lo = [], 0
    for s in range(stages):
        hi = lo + base + (1 if s < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


@dataclass
class MicroBatch:
    ids: Tensor          # [T] packed tokens
    positions: Tensor    # [T]
    cu: Tensor           # [n + 1] int32
    max_len: int
    targets: Tensor      # [T] next-token targets (last stage)
    weights: Tensor      # [T] loss weights (last stage)


class PipelineStage:
    """One stage of a Qwen3/Llama ``model`` (all ranks may hold the full
    model object; a stage only runs and differentiates its own layers)."""

    def __init__(self, model, stage: int, stages: int, group=None) -> None:
        self.model, self.stage, self.stages, self.group = model, stage, stages, group
        self.lo, self.hi = split_layers(model.args.num_layers, stages)[stage]
        self.first, self.last = stage == 0, stage == stages - 1
        self.hidden = model.args.hidden_size

    def params(self) -> list:
        names = [f"layers.{i}." for i in range(self.lo, self.hi)]
        out = [p for n, p in self.model.named_flat_params() if any(n.startswith(x) for x in names)]
        if self.first:
            out.append(self.model.p("embed"))
        if self.last:
            out.append(self.model.p("norm"))
            if not self.model.args.tie_word_embeddings:
                out.append(self.model.p("lm_head"))
        return out

    def sync_tied_embedding_grad(self, ends_group) -> None:
        """With tied input/output embeddings the first stage (embedding) and the
        last stage (LM head) each hold part of the shared weight's gradient;
        sum them over ``ends_group`` (the 2-rank group of the two ends, made by
        ``embedding_group`` on every rank).  Other stages return at once."""
        if not self.model.args.tie_word_embeddings or self.stages == 1 or not (self.first or self.last):
            return
        w = self.model.p("embed")
        g = getattr(w, "main_grad", None)
        if g is None:
            if w.grad is None:
                w.grad = torch.zeros_like(w)
            g = w.grad
        dist.all_reduce(g, group=ends_group)

    def forward(self, mb: MicroBatch, x: Optional[Tensor]) -> Tensor:
        from lumenrl_b200.models.qwen3 import embed
        m = self.model
        if self.first:
            x = embed(mb.ids, m.p("embed"))
        for i in range(self.lo, self.hi):
            x = m._layer(i, x, mb.positions, mb.cu, mb.max_len)
        return x

    def loss(self, mb: MicroBatch, x: Tensor) -> Tensor:
        from lumenrl_b200 import ops
        m = self.model
        h = ops.rmsnorm(x, m.p("norm"), m.args.rms_norm_eps)
        logp, _ = ops.token_logprob(h, m.lm_head, mb.targets, want_entropy=False)
        return -(logp * mb.weights).sum()


def embedding_group(stages: int, ranks: Optional[list] = None):
    """Process group of the first and last pipeline stage (every rank must
    call this, in the same order, as ``dist.new_group`` requires)."""
    ranks = ranks or list(range(stages))
    return dist.new_group([ranks[0], ranks[-1]]) if stages > 1 else None


class OneFOneB:
    """Runs micro-batches through the stages; returns the summed loss on the
    last stage (0 elsewhere).  All stages must call ``run`` with the same
    number of micro-batches; only the first and last stage read the token /
    target fields of each micro-batch, and every stage needs its ``cu`` /
    ``positions`` (attention is per sequence)."""

    def __init__(self, stage: PipelineStage, device: torch.device, dtype: torch.dtype) -> None:
        self.st, self.device, self.dtype = stage, device, dtype
        g = stage.group
        rank = dist.get_rank(g)
        self.prev = dist.get_global_rank(g, rank - 1) if (g is not None and rank > 0) else rank - 1
        self.next = dist.get_global_rank(g, rank + 1) if (g is not None and rank + 1 < stage.stages) else rank + 1

    # -- p2p: a shape message, then the payload; each exchange posts all of
    # its sends and receives in one batch so neighbours never wait on each
    # other's blocking send (Megatron's send_forward_recv_backward pattern)
    def _p2p(self, send_fwd: Optional[Tensor] = None, send_bwd: Optional[Tensor] = None, recv_fwd: bool = False,
             recv_bwd: bool = False) -> tuple[Optional[Tensor], Optional[Tensor]]:
        g, dev = self.st.group, self.device
        sends = [(t, dst) for t, dst in ((send_fwd, self.next), (send_bwd, self.prev)) if t is not None]
        recvs = [src for want, src in ((recv_fwd, self.prev), (recv_bwd, self.next)) if want]
        if not sends and not recvs:
            return None, None
        n_out = [torch.tensor([t.shape[0]], dtype=torch.int64, device=dev) for t, _ in sends]
        n_in = [torch.empty(1, dtype=torch.int64, device=dev) for _ in recvs]
        ops = [dist.P2POp(dist.isend, n, dst, g) for n, (_, dst) in zip(n_out, sends)]
        ops += [dist.P2POp(dist.irecv, n, src, g) for n, src in zip(n_in, recvs)]
        for r in dist.batch_isend_irecv(ops):
            r.wait()
        bufs = [torch.empty(int(n.item()), self.st.hidden, dtype=self.dtype, device=dev) for n in n_in]
        ops = [dist.P2POp(dist.isend, t.contiguous(), dst, g) for t, dst in sends]
        ops += [dist.P2POp(dist.irecv, b, src, g) for b, src in zip(bufs, recvs)]
        for r in dist.batch_isend_irecv(ops):
            r.wait()
        it = iter(bufs)
        x = next(it) if recv_fwd else None
        dy = next(it) if recv_bwd else None
        return x, dy

    def _fwd(self, mb: MicroBatch, x_in: Optional[Tensor], loss_scale: float) -> Tensor:
        st = self.st
        if x_in is not None:
            x_in.requires_grad_(True)
        y = st.forward(mb, x_in)
        return st.loss(mb, y) * loss_scale if st.last else y

    def _bwd(self, x_in: Optional[Tensor], out: Tensor, dy: Optional[Tensor]) -> Optional[Tensor]:
        if self.st.last:
            out.backward()
        else:
            torch.autograd.backward(out, dy)
        return None if self.st.first else x_in.grad

    def run(self, micro_batches: list, loss_scale: float = 1.0) -> float:
        st = self.st
        P, s = st.stages, st.stage
        n = len(micro_batches)
        first, last = st.first, st.last
        warm = min(P - s - 1, n)
        steady = n - warm
        live: list = []
        total = 0.0
        i_f = 0
        for _ in range(warm):
            x, _ = self._p2p(recv_fwd=not first)
            out = self._fwd(micro_batches[i_f], x, loss_scale)
            i_f += 1
            self._p2p(send_fwd=out.detach())
            live.append((x, out))
        x = self._p2p(recv_fwd=not first)[0] if steady > 0 else None
        for i in range(steady):
            out = self._fwd(micro_batches[i_f], x, loss_scale)
            i_f += 1
            if last:
                dy = None
                total += float(out.detach())
            else:
                _, dy = self._p2p(send_fwd=out.detach(), recv_bwd=True)
            live.append((x, out))
            xb, ob = live.pop(0)
            dx = self._bwd(xb, ob, dy)
            if i == steady - 1:
                x = None
                self._p2p(send_bwd=dx)
            else:
                x, _ = self._p2p(send_bwd=dx, recv_fwd=not first)
        while live:
            xb, ob = live.pop(0)
            _, dy = self._p2p(recv_bwd=not last)
            if last:
                total += float(ob.detach())
            dx = self._bwd(xb, ob, dy)
            self._p2p(send_bwd=dx)
        return total
