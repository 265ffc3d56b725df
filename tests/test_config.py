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


def test_kernels_section_overrides_environment(monkeypatch):
    """The config's ``kernels`` section wins over the LRL_* variables and
    rewrites the owning module's switch; None fields change nothing."""
    import importlib

    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.ops.kernel_flags import apply_kernels_config
    ops = importlib.import_module("lumenrl_b200.ops")
    attn = importlib.import_module("lumenrl_b200.ops.attention")
    saved = (ops.DECODE_GEMM, attn.TRAIN_ATTN_BWD)
    monkeypatch.setenv("LRL_DECODE_GEMM", "sk")
    monkeypatch.setenv("LRL_CP_RING", "nvlink")
    try:
        cfg = LumenRLConfig.from_dict({"kernels": {"decode_gemm": "cublas", "train_attn_bwd": "fa2",
                                                   "cp_ring": "pg", "nvls": True}})
        assert cfg.kernels.train_gemm is None
        applied = apply_kernels_config(cfg.kernels)
        assert applied == {"LRL_DECODE_GEMM": "cublas", "LRL_TRAIN_ATTN_BWD": "fa2", "LRL_CP_RING": "pg",
                           "LRL_NVLS": "1"}
        assert ops.DECODE_GEMM == "cublas" and attn.TRAIN_ATTN_BWD == "fa2"
        assert os.environ["LRL_CP_RING"] == "pg"
        with pytest.raises(ValueError):
            apply_kernels_config(LumenRLConfig.from_dict({"kernels": {"decode_attn": "fast"}}).kernels)
    finally:
        ops.DECODE_GEMM, attn.TRAIN_ATTN_BWD = saved
        for k in ("LRL_TRAIN_ATTN_BWD", "LRL_NVLS"):   # set by apply_kernels_config, not by monkeypatch
            os.environ.pop(k, None)
