"""Plugin hooks on CPU: FP8 manager set-up and resets through the vime /
miles hook signatures, rollout through generate_rollout with a fake data
source, and verl registration without verl installed."""

import asyncio
from types import SimpleNamespace

import torch

from lumenrl_b200.engine.inference.engine import RolloutEngine
from lumenrl_b200.models.config import tiny_llama
from lumenrl_b200.models.qwen3 import Qwen3Model
from lumenrl_b200.plugin import hooks, verl


def test_fp8_hooks():
    args = SimpleNamespace(lumenrl_fp8_config={"precision": "fp8"})
    hooks.custom_megatron_init(args)
    assert args._lumenrl_fp8_manager.enabled
    hooks.custom_megatron_before_train_step_hook(args, 0, 0, [torch.nn.Linear(2, 2)], None, None)
    hooks.custom_megatron_before_log_prob_hook(args, torch.nn.Linear(2, 2), "x")
    hooks.custom_megatron_post_save_hook(args, 1, "/tmp/a", "/tmp/b")
    m = hooks.custom_model_provider(True, True, args=SimpleNamespace(lumenrl_model="tiny-llama"))
    assert m.args.num_layers == tiny_llama().num_layers


def test_generate_rollout_and_verl_adapter():
    m = Qwen3Model(tiny_llama(), dtype=torch.float32, requires_grad=False)
    m.init_weights(0)
    eng = RolloutEngine(m, max_num_seqs=8, max_model_len=64, block_size=16, use_cuda_graph=False)

    class Source:
        def get_samples(self, rollout_id):
            return [[[5, 6, 7]] * 4, [[9, 10]] * 2]

    args = SimpleNamespace(_lumenrl_engine=eng, rollout_max_response_len=6, seed=1)
    out = hooks.generate_rollout(args, 0, Source())
    assert [len(g) for g in out["samples"]] == [4, 2]
    r = out["samples"][0][0]
    assert r["prompt_ids"] == [5, 6, 7] and len(r["response_ids"]) == 6 == len(r["logprobs"])
    assert not eng.cache.awake   # the hook hands the GPU memory back
    assert verl.register() is False   # no verl here
    assert "rollout:lumenrl_b200" in verl.PLUGIN_REGISTRY
    ad = verl.RolloutAdapter(engine=eng)
    asyncio.run(ad.resume())
    g = ad.generate_sequences([[1, 2, 3]], n=2, max_new_tokens=4)
    assert g.responses.shape == (2, 4)
    sd = {k: v.clone() for k, v in m.hf_state_dict().items()}
    asyncio.run(ad.update_weights(sd.items()))
    asyncio.run(ad.release())
