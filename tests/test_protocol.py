import pytest
import torch

from lumenrl_b200.core.protocol import DataProto


def mk(n=6):
    return DataProto({"a": torch.arange(n), "b": torch.arange(n * 3).view(n, 3)}, {"m": 1},
                     {"r": [list(range(i)) for i in range(n)]})


def test_select_split_concat_roundtrip():
    d = mk()
    parts = d.split(3)
    assert [len(p) for p in parts] == [2, 2, 2]
    back = DataProto.concat(parts)
    assert torch.equal(back["a"], d["a"]) and back.ragged["r"] == d.ragged["r"]
    sel = d.select_idxs([5, 0])
    assert sel["a"].tolist() == [5, 0] and sel.ragged["r"] == [list(range(5)), []]
    sel2 = d[torch.tensor([True, False, True, False, False, False])]
    assert sel2["a"].tolist() == [0, 2] and sel2.ragged["r"] == [[], [0, 1]]


def test_merge_pads_dim1():
    a = DataProto({"x": torch.ones(2, 3)})
    b = DataProto({"x": torch.ones(1, 5)})
    m = DataProto.merge([a, b])
    assert m["x"].shape == (3, 5) and m["x"][0, 3:].sum() == 0
    with pytest.raises(ValueError):
        DataProto.merge([a, DataProto({"y": torch.ones(1, 2)})])


def test_repeat_and_pad():
    d = mk(3)
    r = d.repeat(2, interleave=True)
    assert r["a"].tolist() == [0, 0, 1, 1, 2, 2] and r.ragged["r"][2] == [0]
    r2 = d.repeat(2, interleave=False)
    assert r2["a"].tolist() == [0, 1, 2, 0, 1, 2]
    p, pad = d.pad_to_divisor(4)
    assert pad == 1 and len(p) == 4 and p["a"][-1] == 0
    assert len(p.unpad(pad)) == 3
    s = d.sample_level_repeat([0, 2, 1])
    assert s["a"].tolist() == [1, 1, 2]


def test_reorder_minibatches_consistency():
    d = mk(5)
    d.reorder([4, 3, 2, 1, 0])
    assert d["a"].tolist() == [4, 3, 2, 1, 0] and d.ragged["r"][0] == [0, 1, 2, 3]
    mbs = list(d.mini_batches(2))
    assert [len(m) for m in mbs] == [2, 2, 1]
    d.check_consistency()
    d.ragged["r"].append([])
    with pytest.raises(ValueError):
        d.check_consistency()


def test_packed_and_router():
    cu = torch.tensor([0, 3, 7])
    d = DataProto.from_packed(torch.arange(7), cu)
    assert d.is_packed and d.max_seqlen == 4 and d.seq_lens.tolist() == [3, 4]
    d2 = mk(2)
    d2.add_router_distributions(3, torch.rand(2, 8))
    assert d2.has_router_distributions() and list(d2.get_router_distributions()) == [3]
