"""Context parallelism: zigzag sequence split and ring attention
(reference ``engine/training/megatron_native_engine.py:1065-1351``: zigzag
``2*CP`` chunks, TE ring attention over ``thd``, log-probs rebuilt with a
differentiable all-reduce).

* ``zigzag_indices(S, cp, rank)``: a sequence is cut into ``2*cp`` equal
  chunks and rank r keeps chunks ``r`` and ``2*cp-1-r``, so every rank gets
  the same amount of causal attention work.
* ``ring_attention(q, k, v, cp_group)``: causal attention of this rank's two
  query chunks against the whole sequence.  The K/V chunks travel round the
  ring (``cp - 1`` point-to-point exchanges, each posted before the block
  computation so the transfer overlaps it); blocks are merged with their
  log-sum-exp.  Per (query chunk, key chunk) pair the mask is all, nothing
  or the causal diagonal, because chunks are ordered.  Backward runs the ring
  again, recomputing each block's probabilities from the global LSE and
  sending each block's dK/dV back with it, so every rank ends with the
  gradient of its own K/V.
* ``gather_seq`` / ``scatter_seq``: put per-rank token tensors back in
  sequence order (all-gather) differentiably, e.g. for log-probs.

Block math: on CUDA with bf16 and head dim 128 every block runs on this
package's tcgen05 flash kernels (``csrc/attn/fa_fwd.cu`` / ``fa_bwd.cu``,
causal for the diagonal blocks, unmasked for the others; the forward returns
the block's LSE, the backward takes the merged output and LSE); other CUDA
shapes use PyTorch's varlen flash-attention kernels; on CPU an fp32
restatement is used.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor


def make_dp_cp_groups(cp: int):
    """Context-parallel groups of ``cp`` consecutive ranks (every rank calls
    this, same order).  Returns this rank's CP group; with ``set_state`` the
    rank's ``ParallelState`` gets ``cp_size``, ``cp_rank`` and ``cp_group``,
    which ``ActorEngine`` and ``SFTTrainer`` read."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % cp:
        raise ValueError(f"world {world} is not a multiple of cp {cp}")
    mine = None
    for g0 in range(0, world, cp):
        g = dist.new_group(list(range(g0, g0 + cp)))
        if g0 <= rank < g0 + cp:
            mine = g
    return mine


def zigzag_indices(S: int, cp: int, rank: int, device=None) -> Tensor:
    if S % (2 * cp):
        raise ValueError(f"sequence length {S} must be a multiple of 2 * cp = {2 * cp}")
    c = S // (2 * cp)
    a = torch.arange(rank * c, (rank + 1) * c, device=device)
    b = torch.arange((2 * cp - 1 - rank) * c, (2 * cp - rank) * c, device=device)
    return torch.cat([a, b])


def _chunk_ids(cp: int, rank: int) -> tuple[int, int]:
    return rank, 2 * cp - 1 - rank


# --------------------------------------------------------------------- block kernels
def _expand(k: Tensor, hq: int) -> Tensor:
    return k if k.shape[1] == hq else k.repeat_interleave(hq // k.shape[1], dim=1)


def _block_fwd(q: Tensor, k: Tensor, v: Tensor, causal: bool, scale: float) -> tuple[Tensor, Tensor]:
    """q [B,H,Tq,D], k/v [B,Hk,Tk,D] -> (o [B,H,Tq,D] in q's dtype, lse [B,H,Tq] fp32)."""
    H = q.shape[1]
    if _tc_ok(q):
        return _tc_fwd(q, k, v, causal, scale)
    if q.is_cuda:
        return _varlen_fwd(q, k, v, causal, scale)
    k, v = _expand(k, H), _expand(v, H)
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if causal:
        Tq, Tk = s.shape[-2], s.shape[-1]
        s = s.masked_fill(torch.ones(Tq, Tk, dtype=torch.bool).triu(1 + Tk - Tq), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.exp(s - lse.unsqueeze(-1)) @ v.float()
    return o.to(q.dtype), lse


def _block_bwd(do: Tensor, q: Tensor, k: Tensor, v: Tensor, o: Tensor, lse: Tensor, causal: bool,
               scale: float) -> tuple[Tensor, Tensor, Tensor]:
    """Gradients of one block given the GLOBAL output ``o`` and ``lse``."""
    H, Hk = q.shape[1], k.shape[1]
    if _tc_ok(q):
        return _tc_bwd(do, q, k, v, o, lse, causal, scale)
    if q.is_cuda:
        return _varlen_bwd(do, q, k, v, o, lse, causal, scale)
    ke, ve = _expand(k, H), _expand(v, H)
    s = (q.float() @ ke.float().transpose(-1, -2)) * scale
    if causal:
        Tq, Tk = s.shape[-2], s.shape[-1]
        s = s.masked_fill(torch.ones(Tq, Tk, dtype=torch.bool).triu(1 + Tk - Tq), float("-inf"))
    p = torch.exp(s - lse.unsqueeze(-1))
    dof = do.float()
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ ve.float().transpose(-1, -2)
    delta = (dof * o.float()).sum(-1, keepdim=True)
    ds = p * (dp - delta) * scale
    dq = ds @ ke.float()
    dk = ds.transpose(-1, -2) @ q.float()
    if Hk != H:
        g = H // Hk
        dk = dk.view(dk.shape[0], Hk, g, *dk.shape[2:]).sum(2)
        dv = dv.view(dv.shape[0], Hk, g, *dv.shape[2:]).sum(2)
    return dq.float(), dk.float(), dv.float()


def _to_thd(x: Tensor) -> Tensor:
    B, H, T, D = x.shape
    return x.transpose(1, 2).reshape(B * T, H, D).contiguous()


def _from_thd(x: Tensor, B: int) -> Tensor:
    T = x.shape[0] // B
    return x.view(B, T, x.shape[1], x.shape[2]).transpose(1, 2)


def _cu(B: int, T: int, dev) -> Tensor:
    return torch.arange(0, (B + 1) * T, T, dtype=torch.int32, device=dev)


def _lse_to_bht(lse: Tensor, B: int, T: int) -> Tensor:
    # the varlen kernel returns [H, B*T] (older builds [B, H, T])
    return lse if lse.dim() == 3 else lse.view(lse.shape[0], B, T).permute(1, 0, 2)


def _varlen_fwd(q, k, v, causal, scale):
    """Flash-attention varlen forward of a [B, H, T, D] block (native GQA)."""
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    out, lse, _seed, _off, _ = torch.ops.aten._flash_attention_forward(
        _to_thd(q), _to_thd(k), _to_thd(v), _cu(B, Tq, q.device), _cu(B, Tk, q.device), Tq, Tk, 0.0, causal, False,
        scale=scale)
    _LSE_LAYOUT[0] = lse.dim()
    return _from_thd(out, B), _lse_to_bht(lse.float(), B, Tq)


def _varlen_bwd(do, q, k, v, o, lse, causal, scale):
    """Block gradients from the GLOBAL output and LSE (fp32 results)."""
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    lse_in = lse.contiguous() if _LSE_LAYOUT[0] == 3 else lse.permute(1, 0, 2).reshape(H, B * Tq).contiguous()
    zero = torch.zeros((), dtype=torch.int64, device=q.device)
    dq, dk, dv = torch.ops.aten._flash_attention_backward(
        _to_thd(do), _to_thd(q), _to_thd(k), _to_thd(v), _to_thd(o.to(q.dtype)), lse_in, _cu(B, Tq, q.device),
        _cu(B, Tk, q.device), Tq, Tk, 0.0, causal, zero, zero, scale=scale)
    return (_from_thd(dq, B).float(), _from_thd(dk, B).float(), _from_thd(dv, B).float())


_LSE_LAYOUT = [2]


def _tc_ok(q: Tensor) -> bool:
    from lumenrl_b200.ops.attention import TRAIN_ATTN
    return TRAIN_ATTN == "tc" and q.is_cuda and q.dtype == torch.bfloat16 and q.shape[-1] == 128


def _tc_fwd(q, k, v, causal, scale):
    """One block on the tcgen05 forward: (o [B,H,T,D] bf16, lse [B,H,T] fp32)."""
    from lumenrl_b200.ops.ext import ext
    B, H, Tq, D = q.shape
    out, lse = ext().fa_fwd(_to_thd(q), _to_thd(k), _to_thd(v), _cu(B, Tq, q.device), Tq, scale, causal=causal)
    return _from_thd(out, B), lse.view(H, B, Tq).permute(1, 0, 2)


def _tc_bwd(do, q, k, v, o, lse, causal, scale):
    """Block gradients on the tcgen05 backward from the GLOBAL output and LSE."""
    from lumenrl_b200.ops.ext import ext
    B, H, Tq, D = q.shape
    lse_in = lse.permute(1, 0, 2).reshape(H, B * Tq).contiguous().float()
    dq, dk, dv = ext().fa_bwd(_to_thd(do.to(q.dtype)), _to_thd(q), _to_thd(k), _to_thd(v), _to_thd(o.to(q.dtype)),
                              lse_in, _cu(B, Tq, q.device), Tq, scale, causal=causal)
    return _from_thd(dq, B).float(), _from_thd(dk, B).float(), _from_thd(dv, B).float()


def _merge(o: Optional[Tensor], lse: Optional[Tensor], ob: Tensor, lb: Tensor) -> tuple[Tensor, Tensor]:
    if o is None:
        return ob.float(), lb
    m = torch.maximum(lse, lb)
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    a, b = torch.exp(lse - m), torch.exp(lb - m)
    new = torch.log(a + b) + m
    wa = (a / (a + b)).unsqueeze(-1)
    return o * wa + ob.float() * (1 - wa), new


# --------------------------------------------------------------------- ring
def _ring_exchange(tensors: list, group, rank: int, cp: int) -> list:
    """Send ``tensors`` to the next rank and receive the previous rank's."""
    nxt, prv = (rank + 1) % cp, (rank - 1) % cp
    g_nxt = dist.get_global_rank(group, nxt) if group is not None else nxt
    g_prv = dist.get_global_rank(group, prv) if group is not None else prv
    recv = [torch.empty(t.shape, dtype=t.dtype, device=t.device) for t in tensors]
    ops = [dist.P2POp(dist.isend, t.contiguous(), g_nxt, group) for t in tensors]
    ops += [dist.P2POp(dist.irecv, r, g_prv, group) for r in recv]
    reqs = dist.batch_isend_irecv(ops)
    return recv, reqs


_FREE = 64          # signal words: [0, 64) ready flags of my slots, [64, 128) free flags of the next rank's slots
_EPOCH_STRIDE = 8   # ready epochs of a slot's lap L are L*8 + 1 .. L*8 + K (K <= 8 tensors per exchange), so
                    # they grow monotonically whatever K each exchange has (2 forward, 4 backward)


def _r256(n: int) -> int:
    return (n + 255) // 256 * 256


class _NVLinkRing:
    """Ring exchange over NVLink for the CP group (instead of NCCL send/recv).

    Every rank owns ``nslots`` receive slots in a CUDA-IPC symmetric buffer.
    ``exchange`` pushes this rank's tensors into the next rank's slot with
    ``p2p_push`` (plain peer stores; push k of the slot's lap L publishes
    epoch 8 L + k + 1 in the slot's ready flag, so the last push's epoch
    implies all) on a side stream, so the transfer overlaps the caller's attention work, and
    waits on the current stream for the previous rank's pushes into this
    rank's slot.  ``release`` hands the slot back (stream-ordered after every
    reader of it, including this rank's own push of its contents) by writing
    the lap into the previous rank's free flag; a push waits for that flag
    before reusing a slot.  Every wait is bounded and reports a status code
    (``check`` raises ``CommTimeout``)."""

    def __init__(self, group, slot_bytes: int, nslots: int = 2, wait_seconds: float = 10.0) -> None:
        from lumenrl_b200.ops.ext import ext
        from lumenrl_b200.parallel.symm import SymmetricBuffer
        self.group = group
        self.cp, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.nxt, self.prv = (self.rank + 1) % self.cp, (self.rank - 1) % self.cp
        self.slot_bytes, self.nslots = _r256(slot_bytes), nslots
        self._e = ext()
        self.data = SymmetricBuffer(self.slot_bytes * nslots // 4, torch.int32, self.rank, self.cp, group)
        self.sig = SymmetricBuffer(128, torch.int32, self.rank, self.cp, group)
        dev = self.data.tensor.device
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.wait_cycles = int(wait_seconds * 2.0e9)
        self.count = 0
        self.side = torch.cuda.Stream(device=dev)
        dist.barrier(group=group)

    def exchange(self, tensors: list) -> tuple[list, tuple]:
        e = self._e
        i, K = self.count, len(tensors)
        if K > _EPOCH_STRIDE:
            raise ValueError("CP ring exchange: at most 8 tensors per exchange")
        self.count += 1
        slot, lap = i % self.nslots, i // self.nslots
        base = slot * self.slot_bytes
        tensors = [t.contiguous() for t in tensors]
        main = torch.cuda.current_stream()
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            if lap > 0:   # the next rank has released this slot's previous contents
                e.p2p_wait(self.sig.ptrs[self.rank] + 4 * (_FREE + slot), lap, self.status, 1, self.wait_cycles)
            off = 0
            for k, t in enumerate(tensors):
                t.record_stream(self.side)
                e.p2p_push(t.view(-1), self.data.ptrs[self.nxt] + base + off, self.sig.ptrs[self.nxt] + 4 * slot,
                           lap * _EPOCH_STRIDE + k + 1, self.counter)
                off += _r256(t.numel() * t.element_size())
        # the previous rank's pushes into this rank's slot (the last one implies all)
        e.p2p_wait(self.sig.ptrs[self.rank] + 4 * slot, lap * _EPOCH_STRIDE + K, self.status, 2, self.wait_cycles)
        mem = self.data.tensor.view(torch.uint8)
        out, off = [], 0
        for t in tensors:
            nb = t.numel() * t.element_size()
            out.append(mem[base + off: base + off + nb].view(t.dtype).view(t.shape))
            off += _r256(nb)
        return out, (slot, lap)

    def release(self, ticket: tuple) -> None:
        torch.cuda.current_stream().wait_stream(self.side)   # this rank's push of the slot has finished
        slot, lap = ticket
        self._e.p2p_signal(self.sig.ptrs[self.prv] + 4 * (_FREE + slot), lap + 1)

    def check(self) -> None:
        s = int(self.status.item())
        if s:
            from lumenrl_b200.parallel.symm import CommTimeout
            raise CommTimeout(f"CP ring exchange: a bounded wait expired (code {s})")

    def close(self) -> None:
        torch.cuda.synchronize()
        self.data.close()
        self.sig.close()


_RINGS: dict = {}


def _nvlink_ring(group, payload_bytes: int) -> Optional[_NVLinkRing]:
    """The group's NVLink ring channel (grown to the payload collectively:
    every rank asks for the same size at the same call), or None when the
    exchange runs over the process group (CPU / gloo, or LRL_CP_RING=pg)."""
    import os
    if os.environ.get("LRL_CP_RING", "nvlink") != "nvlink" or not torch.cuda.is_available():
        return None
    if dist.get_backend(group) != "nccl":
        return None
    key = id(group) if group is not None else 0
    ring = _RINGS.get(key)
    if ring is None or ring.slot_bytes < payload_bytes:
        if ring is not None:
            ring.close()
        ring = _NVLinkRing(group, max(payload_bytes, 1 << 20))
        _RINGS[key] = ring
    return ring


def _payload(tensors: list) -> int:
    return sum(_r256(t.numel() * t.element_size()) for t in tensors)


def _pairs(cp: int, rank: int, src: int):
    """(local q chunk slot, kv chunk slot of `src`, causal?) for every
    (query chunk, key chunk) pair that is not fully masked."""
    qc = _chunk_ids(cp, rank)
    kc = _chunk_ids(cp, src)
    out = []
    for qi, qid in enumerate(qc):
        for ki, kid in enumerate(kc):
            if kid < qid:
                out.append((qi, ki, False))
            elif kid == qid:
                out.append((qi, ki, True))
    return out


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, group, scale):
        cp, rank = dist.get_world_size(group), dist.get_rank(group)
        B, H, T2, D = q.shape
        c = T2 // 2
        qs = [q[:, :, :c], q[:, :, c:]]
        o = [None, None]
        lse = [None, None]
        kv = (k, v)
        ring = _nvlink_ring(group, 3 * _payload([k, v])) if k.is_cuda else None   # 3x: the backward's payload
        ticket = None
        for step in range(cp):
            src = (rank - step) % cp
            reqs = None
            nt = None
            if step < cp - 1:
                if ring is not None:
                    nxt_kv, nt = ring.exchange(list(kv))
                else:
                    nxt_kv, reqs = _ring_exchange(list(kv), group, rank, cp)
            kk, vv = kv
            ks, vs = [kk[:, :, :c], kk[:, :, c:]], [vv[:, :, :c], vv[:, :, c:]]
            for qi, ki, causal in _pairs(cp, rank, src):
                ob, lb = _block_fwd(qs[qi], ks[ki], vs[ki], causal, scale)
                o[qi], lse[qi] = _merge(o[qi], lse[qi], ob, lb)
            if ring is not None and ticket is not None:
                ring.release(ticket)          # the slot just computed from (and pushed on)
            if reqs is not None:
                for r in reqs:
                    r.wait()
            if step < cp - 1:
                kv, ticket = tuple(nxt_kv), nt
        out = torch.cat([o[0], o[1]], 2).to(q.dtype)
        L = torch.cat([lse[0], lse[1]], 2)
        ctx.save_for_backward(q, k, v, out, L)
        ctx.group, ctx.scale = group, scale
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, L = ctx.saved_tensors
        group, scale = ctx.group, ctx.scale
        cp, rank = dist.get_world_size(group), dist.get_rank(group)
        c = q.shape[2] // 2
        sl = [slice(0, c), slice(c, 2 * c)]
        do = do.contiguous()
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        # the K/V block and its gradient travel together round the ring
        kk, vv = k, v
        dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
        dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
        ring = _nvlink_ring(group, _payload([k, v, dk, dv])) if k.is_cuda else None
        ticket = None
        for step in range(cp):
            src = (rank - step) % cp
            for qi, ki, causal in _pairs(cp, rank, src):
                gq, gk, gv = _block_bwd(do[:, :, sl[qi]], q[:, :, sl[qi]], kk[:, :, sl[ki]], vv[:, :, sl[ki]],
                                        out[:, :, sl[qi]], L[:, :, sl[qi]], causal, scale)
                dq[:, :, sl[qi]] += gq
                dk[:, :, sl[ki]] += gk
                dv[:, :, sl[ki]] += gv
            # pass (K, V, dK, dV) on; after cp steps every block is home again
            if ring is not None:
                recv, nt = ring.exchange([kk, vv, dk, dv])
                if ticket is not None:
                    ring.release(ticket)
                ticket = nt
            else:
                recv, reqs = _ring_exchange([kk, vv, dk, dv], group, rank, cp)
                for r in reqs:
                    r.wait()
            kk, vv, dk, dv = recv
        grads = dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
        if ring is not None and ticket is not None:
            ring.release(ticket)             # after the copies above read the home slot
        return (*grads, None, None)


def ring_attention(q: Tensor, k: Tensor, v: Tensor, group=None, scale: Optional[float] = None) -> Tensor:
    """Causal attention for this rank's zigzag chunks.  q [B,H,2c,D] and
    k/v [B,Hk,2c,D] hold chunks (rank, 2cp-1-rank) of each sequence."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if dist.get_world_size(group) == 1:
        from torch.nn.functional import scaled_dot_product_attention as sdpa
        H = q.shape[1]
        return sdpa(q, _expand(k, H), _expand(v, H), is_causal=True, scale=scale)
    return _RingAttention.apply(q, k, v, group, scale)


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, S, group):
        cp, rank = dist.get_world_size(group), dist.get_rank(group)
        parts = [torch.empty_like(x) for _ in range(cp)]
        dist.all_gather(parts, x.contiguous(), group=group)
        out = x.new_empty((S,) + tuple(x.shape[1:]))
        for r in range(cp):
            out[zigzag_indices(S, cp, r, x.device)] = parts[r]
        ctx.S, ctx.group, ctx.rank, ctx.cp = S, group, rank, cp
        return out

    @staticmethod
    def backward(ctx, g):
        # every rank holds the full-sequence gradient of its own use; sum them
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g[zigzag_indices(ctx.S, ctx.cp, ctx.rank, g.device)], None, None


def gather_seq(x_local: Tensor, S: int, group=None) -> Tensor:
    """[2c, ...] zigzag-local rows -> [S, ...] in sequence order on every rank
    (differentiable; the backward sums the ranks' gradients)."""
    return _GatherSeq.apply(x_local, S, group)


def scatter_seq(x: Tensor, group=None) -> Tensor:
    """[S, ...] -> this rank's zigzag rows."""
    cp, rank = dist.get_world_size(group), dist.get_rank(group)
    return x[zigzag_indices(x.shape[0], cp, rank, x.device)]
