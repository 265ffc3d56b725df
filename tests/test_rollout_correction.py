import math

import pytest
import torch

from lumenrl_b200.algorithms import rollout_correction as rc
from lumenrl_b200.core.config import RolloutCorrectionConfig
from lumenrl_b200.core.protocol import DataProto


def test_legacy_tis_mis_known_values():
    out = rc.token_level_tis(torch.tensor([[math.log(10.0)]]), torch.zeros(1, 1), torch.ones(1, 1), clip=2.0)
    assert out.item() == pytest.approx(2.0)
    out = rc.token_level_mis(torch.tensor([[0.0, math.log(2.0)]]), torch.zeros(1, 2), torch.tensor([[3.0, 5.0]]))
    assert out[0].tolist() == pytest.approx([3.0 / 1.5, 5.0 * 2 / 1.5])


def test_token_is_truncation_and_icepop():
    lr = torch.log(torch.tensor([[0.3, 1.0, 5.0]]))
    mask = torch.ones(1, 3)
    w, m = rc.compute_rollout_correction_weights(lr, mask, "token", "2.0")
    assert w[0].tolist() == pytest.approx([0.3, 1.0, 2.0])
    assert m["rollout_is_ratio_fraction_high"] == pytest.approx(1 / 3)
    w, m = rc.compute_rollout_correction_weights(lr, mask, "token", "0.5_4.0")
    assert w[0].tolist() == pytest.approx([0.0, 1.0, 0.0])
    assert m["rollout_is_oob_ratio"] == pytest.approx(2 / 3)


def test_sequence_is_sum_vs_mean():
    lr = torch.tensor([[0.1, 0.1, 0.1, 0.0]])
    mask = torch.tensor([[1.0, 1.0, 1.0, 0.0]])
    w, _ = rc.compute_rollout_correction_weights(lr, mask, "sequence", "10", rollout_is_seq_reduction="sum")
    assert w[0, 0].item() == pytest.approx(math.exp(0.3)) and w[0, 3].item() == 0.0
    w, _ = rc.compute_rollout_correction_weights(lr, mask, "sequence", "10", rollout_is_seq_reduction="mean")
    assert w[0, 0].item() == pytest.approx(math.exp(0.1))


def test_rejection_sampling_criteria():
    lr = torch.tensor([[0.0, 0.0], [1.0, 0.0]])
    mask = torch.ones(2, 2)
    new, m = rc.compute_rollout_rejection_mask(lr, mask, "token_k1", "0.5_2.0")
    # token_k1 = -lr: -1 < log(0.5) -> rejected
    assert new.tolist() == [[1.0, 1.0], [0.0, 1.0]]
    new, _ = rc.compute_rollout_rejection_mask(lr, mask, "seq_max_k2", "0.25")
    assert new.tolist() == [[1.0, 1.0], [0.0, 0.0]]
    new, _ = rc.compute_rollout_rejection_mask(lr, mask, "seq_mean_k3,token_k2", "0.5,0.4")
    assert new[0].tolist() == [1.0, 1.0]
    with pytest.raises(ValueError):
        rc.compute_rollout_rejection_mask(lr, mask, "bogus", "1")


def test_add_to_batch_dealias_and_metrics():
    old = torch.tensor([[-1.0, -2.0, -0.5]])
    roll = torch.tensor([[-1.1, 0.0, -0.4]])  # 0.0 = unreported -> replaced by old
    b = DataProto({"old_log_probs": old, "rollout_log_probs": roll, "response_mask": torch.ones(1, 3)})
    cfg = RolloutCorrectionConfig(rollout_is="token", rollout_is_threshold="2.0", rollout_rs="token_k1",
                                  rollout_rs_threshold="0.5_2.0")
    b, m = rc.compute_rollout_correction_and_add_to_batch(b, cfg)
    assert b["rollout_log_probs"][0, 1].item() == -2.0
    assert "rollout_corr/kl" in m and "rollout_correction/is_weight_mean" in m
    assert b["rollout_is_weights"].shape == (1, 3)


def test_presets_and_bypass():
    assert rc.preset_decoupled_token_icepop().rollout_is_threshold == "0.5_5.0"
    assert rc.preset_bypass_pg_is().loss_type == "reinforce"
    b = DataProto({"rollout_log_probs": torch.ones(1, 2)})
    rc.apply_bypass_mode(b, None)
    assert torch.equal(b["old_log_probs"], b["rollout_log_probs"])


def test_threshold_grammar_shared_by_is_and_rs():
    import pytest as _pt
    from lumenrl_b200.algorithms.rollout_correction import parse_is_threshold, parse_rs_thresholds
    assert parse_is_threshold(2.0) == (2.0, None)
    assert parse_is_threshold("0.5_2") == (2.0, 0.5)
    b = parse_rs_thresholds(["token_k1", "seq_max_k2"], "4, 0.1")
    assert b == {"token_k1": (0.25, 4.0), "seq_max_k2": (None, 0.1)}
    assert parse_rs_thresholds(["seq_sum_k1"], "0.8_1.25") == {"seq_sum_k1": (0.8, 1.25)}
    for bad in ("", "a", "2_1", "0", "-1", "1_2_3"):
        with _pt.raises(ValueError):
            parse_is_threshold(bad)
    with _pt.raises(TypeError):
        parse_is_threshold(True)
    with _pt.raises(ValueError):
        parse_rs_thresholds(["token_k2"], "0.5_2")          # k2 takes an upper bound only
    with _pt.raises(ValueError):
        parse_rs_thresholds(["token_k1", "token_k2", "token_k3"], "1,2")
