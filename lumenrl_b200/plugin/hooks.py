"""Hook functions for driving this framework from the vime / miles RL
frameworks by dotted path (reference ``lumenrl/plugin/vime/hooks.py:28-157``
and ``lumenrl/plugin/miles/hooks.py:36-95``).

    --custom-megatron-init-path   lumenrl_b200.plugin.hooks.custom_megatron_init
    --custom-model-provider-path  lumenrl_b200.plugin.hooks.custom_model_provider
    --rollout-function-path       lumenrl_b200.plugin.hooks.generate_rollout
    --custom-megatron-post-save-hook-path        lumenrl_b200.plugin.hooks.custom_megatron_post_save_hook
    --custom-megatron-before-train-step-hook-path lumenrl_b200.plugin.hooks.custom_megatron_before_train_step_hook
    --custom-megatron-before-log-prob-hook-path   lumenrl_b200.plugin.hooks.custom_megatron_before_log_prob_hook

State travels on the host framework's ``args`` object, as the hook
signatures require:

* ``args.lumenrl_fp8_config`` (dict of ``FP8Config`` fields) ->
  ``custom_megatron_init`` stores an ``FP8TrainingManager`` on
  ``args._lumenrl_fp8_manager``; the before-step / before-log-prob hooks reset
  its per-step state on every model chunk;
* ``args._lumenrl_engine`` (a ``RolloutEngine``) drives ``generate_rollout``:
  the engine wakes, generates every group with ``n = len(group)`` samples of
  one prompt (so the group shares its prompt's KV), and sleeps again.
* ``custom_model_provider`` returns this framework's Qwen3 model for
  ``args.lumenrl_model`` (a preset name) instead of a Megatron ``GPTModel``.
"""

from __future__ import annotations

import logging
from typing import Any

logger = logging.getLogger(__name__)


def custom_megatron_init(args: Any) -> None:
    cfg = getattr(args, "lumenrl_fp8_config", None)
    if cfg is None:
        logger.info("lumenrl_b200: no lumenrl_fp8_config on args; FP8 training stays off")
        return
    from lumenrl_b200.quant.fp8 import FP8Config, FP8TrainingManager
    fp8 = FP8Config(**cfg) if isinstance(cfg, dict) else cfg
    args._lumenrl_fp8_manager = FP8TrainingManager(fp8)


def custom_model_provider(pre_process: bool = True, post_process: bool = True, vp_stage: Any = None,
                          args: Any = None):
    """Builds the Qwen3 model named by ``args.lumenrl_model`` (whole model: this
    framework stages pipelines itself, so pre/post_process must both be set)."""
    if not (pre_process and post_process):
        raise ValueError("lumenrl_b200 models are not split by the host framework's pipeline stages")
    import torch
    from lumenrl_b200.models.config import resolve_model
    from lumenrl_b200.models.qwen3 import Qwen3Model
    name = getattr(args, "lumenrl_model", "qwen3-8b") if args is not None else "qwen3-8b"
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    m = Qwen3Model(resolve_model(name), device=dev, dtype=torch.bfloat16 if dev == "cuda" else torch.float32)
    mgr = getattr(args, "_lumenrl_fp8_manager", None) if args is not None else None
    if mgr is not None:
        m.fp8_manager = mgr
    return m


def _reset_fp8(args: Any, model: Any) -> None:
    mgr = getattr(args, "_lumenrl_fp8_manager", None)
    if mgr is None or not hasattr(mgr, "reset_fp8_state"):
        return
    for chunk in (model if isinstance(model, (list, tuple)) else [model]):
        mgr.reset_fp8_state(chunk)


def custom_megatron_post_save_hook(args: Any, rollout_id: int, checkpoint_dir: str, hf_checkpoint_dir: str) -> None:
    logger.debug("lumenrl_b200: post-save hook rollout %d -> %s", rollout_id, checkpoint_dir)


def custom_megatron_before_train_step_hook(args: Any, rollout_id: int, step_id: int, model: Any, optimizer: Any,
                                           opt_param_scheduler: Any) -> None:
    _reset_fp8(args, model)


def custom_megatron_before_log_prob_hook(args: Any, model: Any, store_prefix: str) -> None:
    _reset_fp8(args, model)


def generate_rollout(args: Any, rollout_id: int, data_source: Any, evaluation: bool = False) -> dict:
    """Returns ``{"samples": [[{prompt_ids, response_ids, logprobs}, ...], ...]}``
    grouped as ``data_source.get_samples(rollout_id)`` groups its prompts (each
    prompt given as token ids, or as an object with ``prompt_ids``)."""
    eng = getattr(args, "_lumenrl_engine", None)
    if eng is None:
        raise RuntimeError("args._lumenrl_engine is not set: create a RolloutEngine and put it on args first")
    from lumenrl_b200.engine.inference.engine import SamplingParams
    groups = data_source.get_samples(rollout_id)
    max_new = int(getattr(args, "rollout_max_response_len", 1024))
    temp = 0.0 if evaluation else float(getattr(args, "rollout_temperature", 1.0))
    eng.wake()
    out = []
    try:
        for gi, group in enumerate(groups):
            ids = [list(getattr(s, "prompt_ids", s)) for s in group]
            if any(p != ids[0] for p in ids):
                raise ValueError("a rollout group must repeat one prompt")
            sp = SamplingParams(max_new_tokens=max_new, temperature=max(temp, 1e-5), n=len(ids),
                                seed=int(getattr(args, "seed", 0)) * 100_003 + rollout_id * 1009 + gi,
                                eos_token_id=getattr(args, "eos_token_id", None))
            g = eng.generate([ids[0]], sp)
            rows = []
            for r in range(len(ids)):
                n = int(g.response_lengths[r])
                rows.append({"prompt_ids": ids[0], "response_ids": g.responses[r, :n].tolist(),
                             "logprobs": g.logprobs[r, :n].tolist()})
            out.append(rows)
    finally:
        eng.sleep()
    return {"samples": out, "evaluation": evaluation}
