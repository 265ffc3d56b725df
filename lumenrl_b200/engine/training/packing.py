"""Sequence packing: remove padding and concatenate rows into one flat
token stream with ``cu_seqlens`` (reference ``lumenrl/engine/training/packing.py:144-353``).

A rollout row is ``prompt ++ response``.  Scoring a response token ``t`` uses
the hidden state at the position before it, so per row we gather hidden rows
``[Lp-1, Lp+Lr-2]`` and targets ``response[0:Lr]``; results scatter back to a
right-padded ``[B, R]`` grid aligned with the response tokens.

``make_micro_batches`` splits rows by a row count or a token budget
(``max_token_len_per_gpu``) with first-fit-decreasing bin packing.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass
class PackedBatch:
    input_ids: Tensor      # [T]
    positions: Tensor      # [T]
    cu_seqlens: Tensor     # [B+1] int32
    max_seqlen: int
    score_index: Tensor    # [N] rows of the hidden stream that score a response token
    targets: Tensor        # [N] target token ids
    out_row: Tensor        # [N] batch row of each scored token
    out_col: Tensor        # [N] response column of each scored token
    rows: list[int]        # batch rows in this pack
    num_rows: int

    def scatter(self, values: Tensor, width: int) -> Tensor:
        out = torch.zeros(self.num_rows, width, dtype=values.dtype, device=values.device)
        out[self.out_row, self.out_col] = values
        return out

    def gather(self, grid: Tensor) -> Tensor:
        """[num_rows, R] grid (rows in this pack's order) -> [N] per scored token."""
        return grid[self.out_row, self.out_col]


def _to_device(x: Tensor, device) -> Tensor:
    """Host index tensors reach the GPU through pinned memory without a
    stream synchronisation (a pageable copy would wait for the queue)."""
    if x.device.type == "cpu" and torch.device(device).type == "cuda":
        return x.pin_memory().to(device, non_blocking=True)
    return x.to(device)


def pack_rows(prompts: list[Tensor], responses: list[Tensor], device, rows: list[int] | None = None) -> PackedBatch:
    """prompts/responses: 1-D token tensors per row (no padding)."""
    ids, pos, cu = [], [], [0]
    score, tgt, orow, ocol = [], [], [], []
    off = 0
    for r, (p, a) in enumerate(zip(prompts, responses)):
        lp, la = int(p.numel()), int(a.numel())
        seq = torch.cat([p, a])
        ids.append(seq)
        pos.append(torch.arange(lp + la))
        if la > 0:
            score.append(torch.arange(off + lp - 1, off + lp + la - 1))
            tgt.append(a)
            orow.append(torch.full((la,), r, dtype=torch.long))
            ocol.append(torch.arange(la))
        off += lp + la
        cu.append(off)
    cat = lambda xs, dt=torch.long: _to_device(torch.cat(xs) if xs else torch.zeros(0, dtype=dt), device)  # noqa: E731
    lens = [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    return PackedBatch(
        input_ids=cat(ids), positions=cat(pos), cu_seqlens=_to_device(torch.tensor(cu, dtype=torch.int32), device),
        max_seqlen=max(lens) if lens else 0, score_index=cat(score), targets=cat(tgt), out_row=cat(orow),
        out_col=cat(ocol), rows=list(rows) if rows is not None else list(range(len(prompts))),
        num_rows=len(prompts))


def pack_rows_cp(prompts: list[Tensor], responses: list[Tensor], device, rows: list[int] | None, cp: int,
                 cp_rank: int) -> PackedBatch:
    """Context-parallel pack: every sequence is right-padded to one length L
    (a multiple of 2 * cp) and this rank keeps its two zigzag chunks of each
    (chunks ``cp_rank`` and ``2 cp - 1 - cp_rank`` of ``2 cp``), so the pack is
    B equal segments of 2 L / (2 cp) tokens at their global positions.  Only
    the response tokens scored by this rank's positions appear in
    ``score_index`` / ``targets`` / ``out_row`` / ``out_col``; pad tokens are
    attended by nothing real (they sit after every real token)."""
    from lumenrl_b200.parallel.context_parallel import zigzag_indices
    lens = [int(p.numel()) + int(a.numel()) for p, a in zip(prompts, responses)]
    L = max(lens) if lens else 0
    L = max(2 * cp, -(-L // (2 * cp)) * (2 * cp))
    loc = zigzag_indices(L, cp, cp_rank)                  # global positions kept here
    two_c = int(loc.numel())
    where = torch.full((L,), -1, dtype=torch.long)
    where[loc] = torch.arange(two_c)
    ids, score, tgt, orow, ocol = [], [], [], [], []
    for r, (p, a) in enumerate(zip(prompts, responses)):
        lp, la = int(p.numel()), int(a.numel())
        seq = torch.zeros(L, dtype=torch.long)
        seq[: lp + la] = torch.cat([p, a]).long()
        ids.append(seq[loc])
        if la > 0:
            g = torch.arange(lp - 1, lp + la - 1)         # positions that score response tokens
            keep = where[g] >= 0
            score.append(r * two_c + where[g[keep]])
            tgt.append(a[keep].long())
            orow.append(torch.full((int(keep.sum()),), r, dtype=torch.long))
            ocol.append(torch.arange(la)[keep])
    B = len(prompts)
    cat = lambda xs: _to_device(torch.cat(xs) if xs else torch.zeros(0, dtype=torch.long), device)  # noqa: E731
    return PackedBatch(
        input_ids=cat(ids), positions=_to_device(loc.repeat(B), device),
        cu_seqlens=torch.arange(0, B * two_c + 1, two_c, dtype=torch.int32, device=device), max_seqlen=two_c,
        score_index=cat(score), targets=cat(tgt), out_row=cat(orow), out_col=cat(ocol),
        rows=list(rows) if rows is not None else list(range(B)), num_rows=B)


def pack_from_grid(prompt_ids: Tensor, prompt_lens, responses: Tensor, response_lens,
                   rows: list[int], device, cp: int = 1, cp_rank: int = 0) -> PackedBatch:
    """Rows of right-padded prompt/response grids -> PackedBatch (with
    ``cp`` > 1: this context-parallel rank's zigzag share, ``pack_rows_cp``).
    The lengths may be tensors or host lists (lists save a device read per
    micro-batch)."""
    pl = prompt_lens if isinstance(prompt_lens, list) else prompt_lens.tolist()
    rl = response_lens if isinstance(response_lens, list) else response_lens.tolist()
    ps = [prompt_ids[r, : pl[r]] for r in rows]
    rs = [responses[r, : rl[r]] for r in rows]
    if cp > 1:
        return pack_rows_cp(ps, rs, device, rows, cp, cp_rank)
    return pack_rows(ps, rs, device, rows)


def make_micro_batches(lengths: list[int], rows_per_micro: int = 0, token_budget: int = 0) -> list[list[int]]:
    """Partition row indices.  ``token_budget`` > 0: first-fit-decreasing bins
    of at most that many tokens (a longer row gets its own bin); otherwise
    consecutive chunks of ``rows_per_micro`` rows."""
    n = len(lengths)
    if token_budget and token_budget > 0:
        order = sorted(range(n), key=lambda i: -lengths[i])
        bins: list[list[int]] = []
        load: list[int] = []
        for i in order:
            for b in range(len(bins)):
                if load[b] + lengths[i] <= token_budget:
                    bins[b].append(i)
                    load[b] += lengths[i]
                    break
            else:
                bins.append([i])
                load.append(lengths[i])
        return [sorted(b) for b in bins]
    k = max(1, rows_per_micro or n)
    return [list(range(a, min(n, a + k))) for a in range(0, n, k)]
