import glob
import os

import pytest

from lumenrl_b200.core.config import LumenRLConfig, RolloutCorrectionConfig

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(HERE, "configs", "*.yaml"))))
def test_repo_recipes_load(path):
    cfg = LumenRLConfig.from_yaml(path)
    assert cfg.algorithm.name in ("grpo", "dapo", "ppo", "opd", "spec_distill")


def test_overrides_and_types():
    cfg = LumenRLConfig.from_dict({"algorithm": {"name": "dapo"}},
                                  ["algorithm.dapo.clip_ratio_high=0.3", "policy.learning_rate=2e-6",
                                   "seed=7", "algorithm.dapo.filter_groups.enable=true"])
    assert cfg.algorithm.dapo.clip_ratio_high == 0.3
    assert cfg.policy.learning_rate == 2e-6 and cfg.seed == 7
    assert cfg.algorithm.dapo.filter_groups.enable is True


def test_unknown_key_rejected():
    with pytest.raises(KeyError):
        LumenRLConfig.from_dict({"policy": {"no_such_key": 1}})


def test_env_interpolation(monkeypatch):
    monkeypatch.setenv("DATA_ROOT", "/data/x")
    cfg = LumenRLConfig.from_dict({"reward": {"dataset": "${oc.env:DATA_ROOT}/train.parquet",
                                              "dataset_split": "${oc.env:MISSING_VAR,test}"},
                                   "checkpointing": {"checkpoint_dir": "${reward.dataset}"}})
    assert cfg.reward.dataset == "/data/x/train.parquet"
    assert cfg.reward.dataset_split == "test"
    assert cfg.checkpointing.checkpoint_dir == "/data/x/train.parquet"


def test_threshold_coercion():
    c = RolloutCorrectionConfig(rollout_is_threshold=2.0, rollout_rs_threshold=0.5)
    assert c.rollout_is_threshold == "2.0" and c.rollout_rs_threshold == "0.5"
    with pytest.raises(ValueError):
        RolloutCorrectionConfig(rollout_is_seq_reduction="max")
