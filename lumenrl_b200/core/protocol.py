"""DataProto: the row-aligned batch container passed between roles.

Behaviour follows the reference's ``lumenrl/core/protocol.py:13-459`` (public
API: same method names and semantics) but the implementation is independent.

A batch has three parts:

* ``tensors`` -- every tensor shares dim 0 (one row per sample);
* ``meta``    -- a dict copied unchanged into every derived batch;
* ``ragged``  -- per-row python payloads (one list entry per row) that are
  re-indexed exactly like tensors (e.g. MoE routed-expert ids, whose per-row
  lengths differ).

Row operations (select/split/concat/merge/repeat/reorder/pad) act on tensors
and ragged columns together so they never fall out of alignment.
"""

from __future__ import annotations

from typing import Any, Iterable, Iterator, Sequence

import torch
import torch.nn.functional as F

_ROUTER_PREFIX = "router_dist_layer_"


class DataProto:
    __slots__ = ("tensors", "meta", "ragged")

    def __init__(self, tensors: dict[str, torch.Tensor] | None = None,
                 meta: dict[str, Any] | None = None,
                 ragged: dict[str, list[Any]] | None = None) -> None:
        self.tensors: dict[str, torch.Tensor] = dict(tensors) if tensors else {}
        self.meta: dict[str, Any] = dict(meta) if meta else {}
        self.ragged: dict[str, list[Any]] = {k: list(v) for k, v in (ragged or {}).items()}

    # ---- construction helpers -------------------------------------------
    def _derive(self, tensors: dict[str, torch.Tensor], rows: Sequence[int] | slice | None) -> "DataProto":
        if rows is None:
            ragged = {k: list(v) for k, v in self.ragged.items()}
        elif isinstance(rows, slice):
            ragged = {k: v[rows] for k, v in self.ragged.items()}
        else:
            ragged = {k: [v[i] for i in rows] for k, v in self.ragged.items()}
        return DataProto(tensors, self.meta.copy(), ragged)

    # ---- packed-sequence helpers -----------------------------------------
    @property
    def cu_seqlens(self) -> torch.Tensor | None:
        return self.tensors.get("cu_seqlens")

    @cu_seqlens.setter
    def cu_seqlens(self, value: torch.Tensor) -> None:
        self.tensors["cu_seqlens"] = value

    @property
    def seq_lens(self) -> torch.Tensor | None:
        return self.tensors.get("seq_lens")

    @seq_lens.setter
    def seq_lens(self, value: torch.Tensor) -> None:
        self.tensors["seq_lens"] = value

    @property
    def max_seqlen(self) -> int:
        if self.seq_lens is not None:
            return int(self.seq_lens.max().item())
        return int(self.meta.get("max_seqlen", 0))

    @property
    def is_packed(self) -> bool:
        return "cu_seqlens" in self.tensors

    # ---- mapping protocol -------------------------------------------------
    def __getitem__(self, item):
        if isinstance(item, str):
            return self.tensors[item]
        return self.select_idxs(item)

    def __setitem__(self, key: str, value: torch.Tensor) -> None:
        self.tensors[key] = value

    def __contains__(self, key: str) -> bool:
        return key in self.tensors

    def __len__(self) -> int:
        for t in self.tensors.values():
            return int(t.shape[0])
        for v in self.ragged.values():
            return len(v)
        return 0

    @property
    def batch_size(self) -> int:
        return len(self)

    def keys(self) -> list[str]:
        return list(self.tensors)

    def check_consistency(self) -> None:
        n = len(self)
        for k, t in self.tensors.items():
            if t.shape[0] != n:
                raise ValueError(f"DataProto has inconsistent batch dimensions: {k} has {t.shape[0]}, expected {n}")
        for k, v in self.ragged.items():
            if len(v) != n:
                raise ValueError(f"DataProto has inconsistent batch dimensions: ragged {k} has {len(v)}, expected {n}")

    # ---- device movement ----------------------------------------------------
    def to(self, device, non_blocking: bool = False) -> "DataProto":
        return self._derive({k: v.to(device, non_blocking=non_blocking) for k, v in self.tensors.items()}, None)

    def cpu(self) -> "DataProto":
        return self.to("cpu")

    def cuda(self, device: int = 0) -> "DataProto":
        return self.to(f"cuda:{device}")

    def pin_memory(self) -> "DataProto":
        return self._derive({k: v.pin_memory() for k, v in self.tensors.items()}, None)

    # ---- row selection ------------------------------------------------------
    def _index(self, idxs) -> torch.Tensor:
        n = len(self)
        if isinstance(idxs, int):
            idx = torch.tensor([idxs + n if idxs < 0 else idxs], dtype=torch.long)
        elif isinstance(idxs, slice):
            idx = torch.arange(n)[idxs]
        elif isinstance(idxs, (list, tuple)):
            idx = torch.as_tensor(list(idxs))
        elif isinstance(idxs, torch.Tensor):
            idx = idxs
        else:
            raise TypeError(f"Unsupported index type for DataProto: {type(idxs)}")
        if idx.dtype == torch.bool:
            if idx.ndim != 1:
                raise ValueError("Boolean index tensor for DataProto must be 1-dimensional")
            if idx.numel() != n:
                raise ValueError(f"Boolean index tensor length mismatch: expected {n}, got {idx.numel()}")
            return idx
        idx = idx.reshape(-1).long()
        return torch.where(idx < 0, idx + n, idx)

    @staticmethod
    def _rows(idx: torch.Tensor) -> list[int]:
        if idx.dtype == torch.bool:
            return idx.nonzero(as_tuple=True)[0].tolist()
        return idx.tolist()

    def select_idxs(self, idxs) -> "DataProto":
        if len(self) == 0:
            return DataProto(meta=self.meta.copy())
        idx = self._index(idxs)
        tensors = {k: v[idx.to(v.device)] for k, v in self.tensors.items()}
        return self._derive(tensors, self._rows(idx))

    def reorder(self, idxs) -> None:
        if len(self) == 0:
            return
        idx = self._index(idxs)
        self.tensors = {k: v[idx.to(v.device)] for k, v in self.tensors.items()}
        rows = self._rows(idx)
        self.ragged = {k: [v[i] for i in rows] for k, v in self.ragged.items()}

    def select(self, keys: list[str]) -> "DataProto":
        return self._derive({k: self.tensors[k] for k in keys if k in self.tensors}, None)

    def update(self, other: "DataProto") -> None:
        self.tensors.update(other.tensors)
        self.ragged.update(other.ragged)
        self.meta.update(other.meta)

    # ---- split / join -------------------------------------------------------
    def split(self, num_chunks: int) -> list["DataProto"]:
        n = len(self)
        if n == 0:
            return [DataProto(meta=self.meta.copy()) for _ in range(num_chunks)]
        out = []
        for i in range(num_chunks):
            lo, hi = i * n // num_chunks, (i + 1) * n // num_chunks
            out.append(self._derive({k: v[lo:hi] for k, v in self.tensors.items()}, slice(lo, hi)))
        return out

    def chunk_sizes(self, sizes: Sequence[int]) -> list["DataProto"]:
        """Split into consecutive chunks of the given row counts."""
        out, lo = [], 0
        for s in sizes:
            hi = lo + int(s)
            out.append(self._derive({k: v[lo:hi] for k, v in self.tensors.items()}, slice(lo, hi)))
            lo = hi
        if lo != len(self):
            raise ValueError(f"chunk sizes sum to {lo}, batch has {len(self)} rows")
        return out

    @staticmethod
    def _join_ragged(parts: list["DataProto"]) -> dict[str, list[Any]]:
        with_ragged = [p for p in parts if p.ragged]
        if not with_ragged:
            return {}
        out: dict[str, list[Any]] = {}
        for key in with_ragged[0].ragged:
            acc: list[Any] = []
            for p in parts:
                acc.extend(p.ragged.get(key, []))
            out[key] = acc
        return out

    @staticmethod
    def concat(protos: list["DataProto"]) -> "DataProto":
        if not protos:
            return DataProto()
        parts = [p for p in protos if len(p) > 0]
        if not parts:
            return DataProto(meta=protos[0].meta.copy())
        keys = parts[0].keys()
        tensors = {k: torch.cat([p.tensors[k] for p in parts], dim=0) for k in keys}
        return DataProto(tensors, parts[0].meta.copy(), DataProto._join_ragged(parts))

    @staticmethod
    def merge(protos: list["DataProto"]) -> "DataProto":
        """Concatenate rows; tensors of rank >= 2 are right-padded with zeros
        along dim 1 to the widest chunk first."""
        if not protos:
            return DataProto()
        parts = [p for p in protos if len(p) > 0]
        if not parts:
            return DataProto(meta=protos[0].meta.copy())
        keys = set(parts[0].keys())
        for i, p in enumerate(parts[1:], start=1):
            ks = set(p.keys())
            if ks != keys:
                raise ValueError(
                    f"DataProto.merge: chunk {i} keys mismatch. missing={keys - ks or '{}'}, extra={ks - keys or '{}'}")
        tensors = {}
        for k in parts[0].keys():
            ts = [p.tensors[k] for p in parts]
            if ts[0].ndim >= 2:
                width = max(t.shape[1] for t in ts)
                ts = [t if t.shape[1] == width else
                      F.pad(t, [0, 0] * (t.ndim - 2) + [0, width - t.shape[1]], value=0) for t in ts]
            tensors[k] = torch.cat(ts, dim=0)
        return DataProto(tensors, parts[0].meta.copy(), DataProto._join_ragged(parts))

    def pad_to_divisor(self, size_divisor: int) -> tuple["DataProto", int]:
        if size_divisor <= 0:
            raise ValueError(f"size_divisor must be positive, got {size_divisor}")
        n = len(self)
        if n == 0:
            return DataProto(meta=self.meta.copy()), 0
        pad = (-n) % size_divisor
        if pad == 0:
            return self._derive({k: v.clone() for k, v in self.tensors.items()}, None), 0
        filler = self.select_idxs(torch.arange(pad) % n)
        return DataProto.concat([self, filler]), pad

    def unpad(self, pad_size: int) -> "DataProto":
        if pad_size < 0:
            raise ValueError(f"pad_size must be non-negative, got {pad_size}")
        if pad_size == 0 or len(self) == 0:
            return self._derive({k: v.clone() for k, v in self.tensors.items()}, None)
        return self.select_idxs(slice(0, max(len(self) - pad_size, 0)))

    def repeat(self, repeat_times: int = 2, interleave: bool = True) -> "DataProto":
        if repeat_times <= 0:
            raise ValueError(f"repeat_times must be positive, got {repeat_times}")
        n = len(self)
        if interleave:
            order = [i for i in range(n) for _ in range(repeat_times)]
        else:
            order = [i for _ in range(repeat_times) for i in range(n)]
        idx = torch.as_tensor(order, dtype=torch.long)
        tensors = {k: v[idx.to(v.device)] for k, v in self.tensors.items()}
        return self._derive(tensors, order)

    def sample_level_repeat(self, repeat_times) -> "DataProto":
        reps = torch.as_tensor(list(repeat_times) if isinstance(repeat_times, tuple) else repeat_times, dtype=torch.long)
        if reps.ndim != 1:
            raise ValueError("repeat_times must be 1-dimensional")
        if reps.numel() != len(self):
            raise ValueError(f"repeat_times length mismatch: expected {len(self)}, got {reps.numel()}")
        if (reps < 0).any():
            raise ValueError("repeat_times values must be non-negative")
        order = [i for i, r in enumerate(reps.tolist()) for _ in range(r)]
        idx = torch.as_tensor(order, dtype=torch.long)
        tensors = {k: v[idx.to(v.device)] for k, v in self.tensors.items()}
        return self._derive(tensors, order)

    def mini_batches(self, batch_size: int) -> Iterator["DataProto"]:
        n = len(self)
        for lo in range(0, n, batch_size):
            hi = min(lo + batch_size, n)
            yield self._derive({k: v[lo:hi] for k, v in self.tensors.items()}, slice(lo, hi))

    # ---- MoE router distributions (legacy logit-replay path) ----------------
    def add_router_distributions(self, layer_idx: int, logits: torch.Tensor) -> None:
        self.tensors[f"{_ROUTER_PREFIX}{layer_idx}"] = logits.detach().cpu()

    def get_router_distributions(self) -> dict[int, torch.Tensor]:
        return {int(k[len(_ROUTER_PREFIX):]): v for k, v in self.tensors.items() if k.startswith(_ROUTER_PREFIX)}

    def has_router_distributions(self) -> bool:
        return any(k.startswith(_ROUTER_PREFIX) for k in self.tensors)

    @classmethod
    def from_packed(cls, packed_input_ids: torch.Tensor, cu_seqlens: torch.Tensor,
                    position_ids: torch.Tensor | None = None,
                    extra_tensors: dict[str, torch.Tensor] | None = None,
                    meta: dict[str, Any] | None = None) -> "DataProto":
        seq_lens = cu_seqlens[1:] - cu_seqlens[:-1]
        tensors = {"input_ids": packed_input_ids, "cu_seqlens": cu_seqlens, "seq_lens": seq_lens}
        if position_ids is not None:
            tensors["position_ids"] = position_ids
        if extra_tensors:
            tensors.update(extra_tensors)
        m = dict(meta or {})
        m["max_seqlen"] = int(seq_lens.max().item()) if seq_lens.numel() else 0
        return cls(tensors=tensors, meta=m)

    def __repr__(self) -> str:
        shapes = {k: tuple(v.shape) for k, v in self.tensors.items()}
        return f"DataProto(rows={len(self)}, tensors={shapes}, ragged={list(self.ragged)}, meta={list(self.meta)})"
