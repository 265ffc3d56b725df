"""Advantage estimators, losses and KL control against closed forms."""

import math

import pytest
import torch

from lumenrl_b200.algorithms import ADV_ESTIMATOR_REGISTRY
from lumenrl_b200.algorithms import losses as L
from lumenrl_b200.algorithms.dapo_sampling import filter_groups_keep_mask, overlong_buffer_penalty
from lumenrl_b200.algorithms.kl_controller import AdaptiveKLController, apply_kl_penalty, kl_penalty_forward, kl_penalty_token
from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.core.registry import ALGORITHM_REGISTRY
from lumenrl_b200.ops import reference as ref


def cfg(g=2):
    c = LumenRLConfig()
    c.algorithm.grpo.num_generations = g
    c.algorithm.dapo.num_generations = g
    return c


def test_grpo_advantage_group_relative():
    b = DataProto({"rewards": torch.tensor([1.0, 3.0, 0.0, 4.0])})
    adv = ALGORITHM_REGISTRY.get("grpo")(cfg(2)).compute_advantages(b)["advantages"].view(-1, 2)
    assert torch.allclose(adv.sum(1), torch.zeros(2), atol=1e-6)
    assert torch.allclose(adv, torch.tensor([[-1.0, 1.0], [-1.0, 1.0]]))   # biased std


def test_dapo_unbiased_std_and_dynamic_mask():
    b = DataProto({"rewards": torch.tensor([1.0, 0.0, 1.0, 1.0])})
    out = ALGORITHM_REGISTRY.get("dapo")(cfg(2)).compute_advantages(b)
    assert torch.allclose(out["advantages"][:2], torch.tensor([1.0, -1.0]) / math.sqrt(2), atol=1e-6)
    assert out["dapo_sample_mask"].tolist() == [1.0, 1.0, 0.0, 0.0]


def test_all_estimators_run_and_shapes():
    c = cfg(4)
    for name, fn in ADV_ESTIMATOR_REGISTRY.items():
        b = DataProto({"rewards": torch.tensor([1.0, 0, 0, 1, 1, 0, 1, 1]), "response_mask": torch.ones(8, 5),
                       "values": torch.rand(8, 5)})
        fn(b, c)
        assert b["advantages"].shape[0] == 8, name
        assert torch.isfinite(b["advantages"]).all(), name


def test_rloo_closed_form():
    b = DataProto({"rewards": torch.tensor([1.0, 0.0, 0.0]), "response_mask": torch.ones(3, 1)})
    c = cfg(3)
    ADV_ESTIMATOR_REGISTRY["rloo_vectorized"](b, c)
    assert torch.allclose(b["advantages"].squeeze(-1), torch.tensor([1.0, -0.5, -0.5]))


def test_gae_matches_loop():
    torch.manual_seed(0)
    v, r = torch.rand(2, 6), torch.tensor([1.0, 0.5])
    mask = torch.ones(2, 6)
    mask[1, 4:] = 0
    c = cfg()
    c.algorithm.ppo.discount, c.algorithm.ppo.gae_lambda = 0.9, 0.8
    b = DataProto({"rewards": r, "values": v, "response_mask": mask})
    ADV_ESTIMATOR_REGISTRY["gae"](b, c)
    # explicit recursion for row 0
    tr = torch.zeros(6)
    tr[5] = 1.0
    adv, run = torch.zeros(6), 0.0
    for t in range(5, -1, -1):
        nv = v[0, t + 1] if t < 5 else 0.0
        run = tr[t] + 0.9 * nv - v[0, t] + 0.9 * 0.8 * run
        adv[t] = run
    assert torch.allclose(b["advantages"][0], adv, atol=1e-5)
    assert (b["advantages"][1, 4:] == 0).all()


def test_policy_gradient_and_asym_clip():
    logp = torch.tensor([[0.0, math.log(2.0)]])
    old = torch.zeros(1, 2)
    adv = torch.tensor([[1.0, 1.0]])
    # ratio 1 and 2; symmetric clip 0.2 -> min(2*1, 1.2*1) = 1.2
    assert L.policy_gradient_loss(logp, old, adv, 0.2).item() == pytest.approx(-(1.0 + 1.2) / 2)
    # asym clip-higher 0.28 -> 1.28
    assert L.asymmetric_clip_loss(logp, old, adv, 0.2, 0.28).item() == pytest.approx(-(1.0 + 1.28) / 2)
    # dual clip: negative advantage with a huge ratio is capped at c * |A|
    big = torch.tensor([[math.log(10.0)]])
    v = L.asymmetric_clip_loss(big, torch.zeros(1, 1), torch.tensor([[-1.0]]), 0.2, 0.28, clip_ratio_c=3.0)
    assert v.item() == pytest.approx(3.0)
    # global-token normalisation
    m = torch.ones(1, 2)
    g = L.asymmetric_clip_loss(logp, old, adv, 0.2, 0.28, mask=m, batch_num_tokens=8, dp_size=2)
    assert g.item() == pytest.approx(-(1.0 + 1.28) / 8 * 2)


def test_fused_loss_definition_matches_library():
    torch.manual_seed(0)
    n = 200
    old = -torch.rand(n)
    logp = old + 0.4 * torch.randn(n)
    adv, mask, w = torch.randn(n), (torch.rand(n) > 0.3).float(), torch.rand(n) * 2
    lib = L.asymmetric_clip_loss(logp, old, adv, 0.2, 0.28, mask=mask, clip_ratio_c=3.0, batch_num_tokens=77,
                                 rollout_is_weights=w)
    fused = ref.ppo_clip_token_loss(logp, old, adv, mask, 0.2, 0.28, 3.0, w, 77.0)
    assert lib.item() == pytest.approx(fused.item(), rel=1e-5)


def test_agg_modes():
    lm = torch.tensor([[1.0, 2.0, 3.0], [4.0, 0.0, 0.0]])
    mask = torch.tensor([[1.0, 1.0, 1.0], [1.0, 0.0, 0.0]])
    assert L.agg_loss(lm, mask, "token-mean").item() == pytest.approx(10 / 4)
    assert L.agg_loss(lm, mask, "seq-mean-token-sum").item() == pytest.approx((6 + 4) / 2)
    assert L.agg_loss(lm, mask, "seq-mean-token-mean").item() == pytest.approx((2 + 4) / 2)
    assert L.agg_loss(lm, mask, "seq-mean-token-sum-norm").item() == pytest.approx((6 + 4) / 2 / 3)


def test_gmpo_and_value_loss():
    lp = torch.tensor([[0.1, -0.1]])
    old = torch.zeros(1, 2)
    adv = torch.ones(1, 2)
    v = L.gmpo_loss(lp, old, adv, 0.4, 0.4, mask=torch.ones(1, 2))
    assert v.item() == pytest.approx(-1.0, abs=1e-6)
    vl = L.value_loss(torch.tensor([1.0]), torch.tensor([0.0]), torch.tensor([0.0]), 0.5)
    assert vl.item() == pytest.approx(1.0)


def test_opd_kl_directions():
    s = torch.randn(2, 3, 11)
    t = torch.randn(2, 3, 11)
    rev = L.opd_kl_divergence(s, t, kl_direction="reverse")
    fwd = L.opd_kl_divergence(s, t, kl_direction="forward")
    ls, lt = s.log_softmax(-1), t.log_softmax(-1)
    assert rev.item() == pytest.approx((ls.exp() * (ls - lt)).sum(-1).mean().item(), rel=1e-5)
    assert fwd.item() == pytest.approx((lt.exp() * (lt - ls)).sum(-1).mean().item(), rel=1e-5)
    assert L.opd_kl_divergence(s, s).item() == pytest.approx(0.0, abs=1e-6)


def test_kl_estimators_and_controller():
    lp, rf = torch.tensor([0.5]), torch.tensor([0.0])
    assert kl_penalty_forward(lp, rf, "k1").item() == pytest.approx(0.5)
    assert kl_penalty_forward(lp, rf, "k2").item() == pytest.approx(0.125)
    assert kl_penalty_forward(lp, rf, "k3").item() == pytest.approx(math.exp(-0.5) + 0.5 - 1)
    x = torch.tensor([0.5], requires_grad=True)
    y = kl_penalty_token(x, rf, "k3+")
    y.backward()
    assert x.grad.item() == pytest.approx(0.5)          # k2 gradient, k3 value
    assert y.item() == pytest.approx(math.exp(-0.5) + 0.5 - 1)
    c = AdaptiveKLController(0.1, 0.01, 100)
    c.update(1.0, 10)
    assert c.value == pytest.approx(0.1 * (1 + 0.2 * 10 / 100))
    b = DataProto({"old_log_probs": torch.zeros(2, 3), "ref_log_probs": torch.zeros(2, 3),
                   "rewards": torch.tensor([1.0, 2.0]), "response_mask": torch.tensor([[1, 1, 0], [1, 1, 1.0]])})
    b, m = apply_kl_penalty(b, c, "kl")
    assert b["rewards"][0].tolist() == [0.0, 1.0, 0.0] and b["rewards"][1, 2] == 2.0


def test_dapo_sampling_helpers():
    pen = overlong_buffer_penalty([10, 18, 20, 22], max_resp_len=20, buffer_len=4, penalty_factor=1.0)
    assert pen.tolist() == pytest.approx([0.0, -0.5, -1.0, -1.5])
    keep, kept = filter_groups_keep_mask([1, 1, 0, 1, 0, 0, 1], ["a", "a", "b", "b", "c", "c", "d"])
    assert keep.tolist() == [False, False, True, True, False, False, True] and kept == ["b", "d"]


def test_grpo_dapo_compute_loss():
    c = cfg(2)
    for name in ("grpo", "dapo", "ppo"):
        b = DataProto({"log_probs": torch.randn(2, 5, requires_grad=True), "old_log_probs": torch.randn(2, 5),
                       "advantages": torch.randn(2), "response_mask": torch.ones(2, 5),
                       "values": torch.randn(2, 5), "returns": torch.randn(2, 5)})
        if name == "ppo":
            b["advantages"] = torch.randn(2, 5)
        loss, m = ALGORITHM_REGISTRY.get(name)(c).compute_loss(b)
        loss.backward()
        assert loss.ndim == 0 and "loss_total" in m
