"""Dispatch / collect semantics between the single controller and its workers.

Modes and their meaning follow ``lumenrl/controller/dispatch.py:11-352``:

===========================  =========================================  ======================
mode                         dispatch                                   collect
===========================  =========================================  ======================
rank_zero                    whole batch to worker 0 only               worker 0's result
one_to_all (alias broadcast) whole batch to every worker                merge (optionally dedup)
all_to_all                   even split, round-robin if short           merge
dp_compute / dp_compute_proto / dp_compute_proto_with_func / dp_compute_metric
                             split by data-parallel group; an N-D       merge (right-pad dim 1)
                             ``mesh_mapping`` routes group ids to
                             workers (TP/PP peers get identical data);
                             the mapping can be cached under a lazy key
direct_rollout_method        forbidden (raises)                         forbidden
===========================  =========================================  ======================
"""

from __future__ import annotations

from enum import Enum
from typing import Any, Callable, Optional

from lumenrl_b200.core.protocol import DataProto


class DispatchMode(str, Enum):
    RANK_ZERO = "rank_zero"
    DP_COMPUTE_PROTO = "dp_compute_proto"
    DP_COMPUTE = "dp_compute"
    DP_COMPUTE_PROTO_WITH_FUNC = "dp_compute_proto_with_func"
    DP_COMPUTE_METRIC = "dp_compute_metric"
    ONE_TO_ALL = "one_to_all"
    ALL_TO_ALL = "all_to_all"
    DIRECT_ROLLOUT_METHOD = "direct_rollout_method"


def normalize_mode(mode) -> DispatchMode:
    if mode is None:
        return DispatchMode.DP_COMPUTE_PROTO
    if isinstance(mode, DispatchMode):
        return mode
    return DispatchMode.ONE_TO_ALL if mode == "broadcast" else DispatchMode(mode)


def _forbidden(*_a, **_k):
    raise RuntimeError("Direct rollout call is forbidden.")


def _split_by_mesh(data: DataProto, n: int, mesh_mapping: Optional[list[int]], lazy_state: Optional[dict],
                   lazy_key: Optional[str]) -> list[DataProto]:
    mapping = mesh_mapping
    if lazy_state is not None and lazy_key is not None:
        cached = lazy_state.get(lazy_key)
        if isinstance(cached, list):
            mapping = cached
        elif mesh_mapping is not None:
            lazy_state[lazy_key] = list(mesh_mapping)
    if mapping is None:
        return data.split(n)
    if len(mapping) != n:
        raise ValueError("mesh_mapping length must equal num_workers.")
    if not mapping:
        return []
    groups = data.split(max(mapping) + 1)
    return [groups[g] for g in mapping]


def _dispatch(mode: DispatchMode) -> Callable[..., list[DataProto]]:
    if mode is DispatchMode.RANK_ZERO:
        return lambda d, n, **_: [d] if n > 0 else []
    if mode is DispatchMode.ONE_TO_ALL:
        return lambda d, n, **_: [d] * n
    if mode is DispatchMode.ALL_TO_ALL:
        def a2a(d, n, **_):
            parts = d.split(n)
            if not parts:
                return [DataProto() for _ in range(n)]
            return [parts[i % len(parts)] for i in range(n)]
        return a2a
    if mode is DispatchMode.DIRECT_ROLLOUT_METHOD:
        return _forbidden
    return lambda d, n, mesh_mapping=None, lazy_state=None, lazy_key=None: _split_by_mesh(
        d, n, mesh_mapping, lazy_state, lazy_key)


def _merge_dedup(results: list[DataProto], deduplicate_by_identity: bool = False) -> DataProto:
    if deduplicate_by_identity:
        seen, uniq = set(), []
        for r in results:
            if id(r) not in seen:
                seen.add(id(r))
                uniq.append(r)
        results = uniq
    return DataProto.merge(results)


def _collect(mode: DispatchMode) -> Callable[..., DataProto]:
    if mode is DispatchMode.RANK_ZERO:
        return lambda rs, **_: rs[0] if rs else DataProto()
    if mode is DispatchMode.DIRECT_ROLLOUT_METHOD:
        return _forbidden
    if mode in (DispatchMode.ONE_TO_ALL, DispatchMode.ALL_TO_ALL):
        return _merge_dedup
    return lambda rs, **_: DataProto.merge(rs)


DISPATCH_MODE_FN_REGISTRY: dict[DispatchMode, dict[str, Callable]] = {
    m: {"dispatch_fn": _dispatch(m), "collect_fn": _collect(m)} for m in DispatchMode
}


def dispatch_proto(data: DataProto, num_workers: int, mode=None, *, mesh_mapping=None, lazy_state=None,
                   lazy_key=None) -> list[DataProto]:
    fn = DISPATCH_MODE_FN_REGISTRY[normalize_mode(mode)]["dispatch_fn"]
    return fn(data, num_workers, mesh_mapping=mesh_mapping, lazy_state=lazy_state, lazy_key=lazy_key)


def collect_proto(results: list[DataProto], mode=None, *, deduplicate_by_identity: bool = False) -> DataProto:
    fn = DISPATCH_MODE_FN_REGISTRY[normalize_mode(mode)]["collect_fn"]
    return fn(results, deduplicate_by_identity=deduplicate_by_identity)


def dispatch_with_dp_ranks(data: DataProto, num_workers: int, dp_rank_mapping: list[int]) -> list[DataProto]:
    """Split by the number of distinct dp ranks; workers sharing a dp rank
    (TP/PP peers) receive the same chunk."""
    if len(dp_rank_mapping) != num_workers:
        raise ValueError(f"dp_rank_mapping length ({len(dp_rank_mapping)}) != num_workers ({num_workers})")
    chunks = data.split(len(set(dp_rank_mapping)))
    return [chunks[r] for r in dp_rank_mapping]


def collect_with_mask(results: list[Any], collect_mask: list[bool]) -> DataProto:
    """Keep only the results of workers that own their output (e.g. TP rank 0
    of each DP group) and merge them."""
    return DataProto.merge([r for r, keep in zip(results, collect_mask) if keep])
