"""MoE router diagnostics and expert resharding (reference behaviour:
``lumenrl/moe/moe_utils.py:143-188``, ``lumenrl/moe/expert_parallel.py``)."""

import math

import torch

from lumenrl_b200.moe.diagnostics import RouterStats, expert_utilization, reshard_experts, router_entropy


def test_router_entropy_uniform_and_peaked():
    E = 8
    uni = torch.full((5, E), 1.0 / E)
    assert abs(float(router_entropy(uni)) - math.log(E)) < 1e-6
    peak = torch.zeros(3, E)
    peak[:, 2] = 1.0
    assert float(router_entropy(peak)) == 0.0


def test_expert_utilization_counts():
    u = expert_utilization(torch.tensor([4.0, 4.0, 0.0, 8.0]))
    assert u["dead_experts"] == 1
    assert abs(u["max_share"] - 0.5) < 1e-12 and u["min_share"] == 0.0
    assert abs(u["max_over_mean"] - 2.0) < 1e-12
    even = expert_utilization(torch.ones(6))
    assert even["cv"] == 0.0 and even["max_over_mean"] == 1.0


def test_router_stats_accumulate_over_layers():
    torch.manual_seed(0)
    st = RouterStats(num_layers=3, num_experts=4, device="cpu")
    probs = torch.softmax(torch.randn(10, 4), -1)
    ids = torch.topk(probs, 2, -1).indices
    st.observe(1, probs, ids)
    st.observe(1, probs, ids)
    s = st.summary()
    assert abs(s["moe/router_entropy"] - float(router_entropy(probs))) < 1e-6
    counts = torch.bincount(ids.reshape(-1), minlength=4).double() * 2
    assert abs(s["moe/expert_max_over_mean"] - expert_utilization(counts)["max_over_mean"]) < 1e-9
    st.reset()
    assert st.summary() == {}


def test_reshard_experts_narrower_and_wider():
    full = torch.arange(8 * 3 * 2).reshape(8, 3, 2)
    train = list(torch.split(full, 2))              # EP 4 training layout, 2 experts per rank
    two = reshard_experts(train, 2)
    assert len(two) == 2 and torch.equal(torch.cat(two), full) and two[0].shape[0] == 4
    eight = reshard_experts(two, 8)
    assert len(eight) == 8 and torch.equal(eight[5], full[5:6])
    try:
        reshard_experts(train, 3)
        raise AssertionError("expected a ValueError")
    except ValueError:
        pass


def test_moe_layer_fills_router_stats_in_training():
    from lumenrl_b200.models.config import tiny_qwen3_moe
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.moe.diagnostics import attach_router_stats
    args = tiny_qwen3_moe()
    m = Qwen3Model(args, device="cpu", dtype=torch.float32, requires_grad=True)
    m.init_weights(0)
    st = attach_router_stats(m)
    T = 12
    ids = torch.randint(0, args.vocab_size, (T,))
    pos = torch.arange(T)
    cu = torch.tensor([0, T], dtype=torch.int32)
    h = m.forward_packed(ids, pos, cu, T)
    h.float().sum().backward()
    s = st.summary()
    n_moe = sum(1 for i in range(args.num_layers) if args.is_moe_layer(i))
    assert n_moe > 0 and s["moe/router_entropy"] > 0
    assert float(st.counts.sum()) == n_moe * T * args.num_experts_per_tok
