"""HTTP rollout replicas: two replica processes behind the load-balancing
client draw the same samples as one in-process engine, and the control calls
(health, drain, sleep / wake, weight reload from safetensors) work."""

import torch

from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
from lumenrl_b200.engine.inference.replicas import HttpRolloutEngine, ReplicaManager, RolloutClient
from lumenrl_b200.models.config import tiny_llama
from lumenrl_b200.models.qwen3 import Qwen3Model

KW = {"max_num_seqs": 8, "max_model_len": 128, "use_cuda_graph": False}


def _local(seed: int, prompts, sp):
    m = Qwen3Model(tiny_llama(), device=torch.device("cpu"), dtype=torch.float32, requires_grad=False)
    m.init_weights(seed)
    return m, RolloutEngine(m, **KW).generate(prompts, sp)


def test_client_split_is_contiguous_and_even():
    c = RolloutClient(["http://a", "http://b", "http://c"])
    assert c.split(7) == [(0, 3), (3, 5), (5, 7)]
    assert c.split(2) == [(0, 1), (1, 2), (2, 2)]
    c.close()


def test_http_replicas_match_one_engine(tmp_path):
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, 2048, (int(n),), generator=g).tolist() for n in (8, 12, 9, 10, 11)]
    sp = SamplingParams(max_new_tokens=8, n=2, seed=7, eos_token_id=None, stop_at_eos=False)
    mgr = ReplicaManager(tiny_llama(), ["cpu", "cpu"], seed=3, engine_kwargs=KW).create()
    try:
        eng = HttpRolloutEngine(mgr)
        assert [h["weight_version"] for h in mgr.client.health()] == [0, 0]
        out = eng.generate(prompts, sp)
        _, ref = _local(3, prompts, sp)
        assert out.responses.shape[0] == ref.responses.shape[0] == 10
        assert torch.equal(out.prompt_index, ref.prompt_index.cpu())
        for i in range(10):
            L = int(ref.response_lengths[i])
            assert int(out.response_lengths[i]) == L
            assert out.responses[i, :L].tolist() == ref.responses[i, :L].tolist()
            assert torch.allclose(out.logprobs[i, :L], ref.logprobs[i, :L].cpu(), atol=1e-4)
        # control plane
        eng.sleep()
        eng.wake()
        mgr.drain_all()
        # new weights through a safetensors file, as a filesystem weight sync writes them
        from safetensors.torch import save_file
        m5 = Qwen3Model(tiny_llama(), device=torch.device("cpu"), dtype=torch.float32, requires_grad=False)
        m5.init_weights(5)
        save_file({k: v.contiguous() for k, v in m5.hf_state_dict().items()}, str(tmp_path / "model.safetensors"))
        assert eng.update_weights_from_path(str(tmp_path)) == [1, 1]
        out5 = eng.generate(prompts, sp)
        _, ref5 = _local(5, prompts, sp)
        for i in range(10):
            L = int(ref5.response_lengths[i])
            assert out5.responses[i, :L].tolist() == ref5.responses[i, :L].tolist()
    finally:
        mgr.shutdown()
