import pytest
import torch

from lumenrl_b200.controller.colocation import create_colocated_worker_cls, resolve_worker_class
from lumenrl_b200.controller.dispatch import (DISPATCH_MODE_FN_REGISTRY, DispatchMode, collect_proto,
                                              dispatch_proto, dispatch_with_dp_ranks)
from lumenrl_b200.controller.worker_group import ResourcePool, WorkerGroup
from lumenrl_b200.core.protocol import DataProto


def test_dispatch_modes():
    p = DataProto({"x": torch.arange(12).view(4, 3).float()})
    ch = dispatch_proto(p, 2)
    assert [c.batch_size for c in ch] == [2, 2]
    assert torch.equal(collect_proto(ch)["x"], p["x"])
    assert all(c.batch_size == 4 for c in dispatch_proto(p, 3, "broadcast"))
    assert len(dispatch_proto(p, 4, DispatchMode.RANK_ZERO)) == 1
    nd = dispatch_proto(DataProto({"x": torch.arange(10)}), 4, mesh_mapping=[0, 0, 1, 1])
    assert torch.equal(nd[0]["x"], nd[1]["x"]) and not torch.equal(nd[0]["x"], nd[2]["x"])
    lazy: dict = {}
    dispatch_proto(p, 2, mesh_mapping=[0, 1], lazy_state=lazy, lazy_key="k")
    assert lazy["k"] == [0, 1]
    assert set(DispatchMode) <= set(DISPATCH_MODE_FN_REGISTRY)
    with pytest.raises(RuntimeError):
        dispatch_proto(p, 2, DispatchMode.DIRECT_ROLLOUT_METHOD)
    d = dispatch_with_dp_ranks(DataProto({"x": torch.arange(4)}), 4, [0, 0, 1, 1])
    assert torch.equal(d[0]["x"], d[1]["x"])
    first, second = DataProto({"x": torch.zeros(2, 1)}), DataProto({"x": torch.ones(2, 1)})
    assert torch.equal(collect_proto([first, second], "rank_zero")["x"], first["x"])


def test_colocation_and_registry():
    class A:
        def __init__(self, **k):
            self.v = 1

        def f(self):
            return "a"

    class B:
        def __init__(self, **k):
            pass

        def f(self):
            return "b"

    C = create_colocated_worker_cls({"actor": A, "ref": B})
    c = C()
    assert c.actor_f() == "a" and c.ref_f() == "b"
    assert resolve_worker_class("actor").__name__ == "ActorWorker"


class Echo:
    def __init__(self, scale=1):
        import os
        self.rank = int(os.environ["RANK"])
        self.scale = scale

    def double(self, d: DataProto) -> DataProto:
        return DataProto({"x": d["x"] * 2 * self.scale})

    def whoami(self):
        return self.rank

    def boom(self):
        raise ValueError("bad")


def test_worker_group_processes():
    pool = ResourcePool("cpu", [2])
    a, b = pool.split([1, 1])
    assert a.gpu_ids == [0] and b.gpu_ids == [1]
    wg = WorkerGroup(Echo, pool, scale=3)
    try:
        assert wg.execute_all_sync("whoami") == [0, 1]
        out = wg.dispatch_and_call("double", DataProto({"x": torch.arange(4)}))
        assert out["x"].tolist() == [0, 6, 12, 18]
        assert all(wg.is_alive())
        with pytest.raises(RuntimeError, match="bad"):
            wg.execute_all_sync("boom")
        assert wg.call_with_timeout("whoami", 30) == [0, 1]
    finally:
        wg.shutdown()
