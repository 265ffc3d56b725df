"""HF ``transformers`` fallback engine: an HF twin of a native Qwen3 model
scores sequences like the native model, generates greedily like the native
forward, rejects incomplete weight syncs, and serves the DataProto
generation interface; the native rollout engine never samples ids past its
vocabulary limit."""

import pytest
import torch

from lumenrl_b200.models.config import tiny_qwen3

transformers = pytest.importorskip("transformers")


def _native():
    from lumenrl_b200.models.qwen3 import Qwen3Model
    m = Qwen3Model(tiny_qwen3(), dtype=torch.float32, requires_grad=False)
    m.init_weights(3)
    return m


def test_hf_twin_log_probs_match_native():
    from lumenrl_b200.engine.inference.hf_engine import HFEngine
    m = _native()
    eng = HFEngine.from_native(m)
    ids = torch.randint(0, m.args.vocab_size, (2, 10), generator=torch.Generator().manual_seed(0))
    lp = eng.compute_log_probs(ids)
    assert lp.shape == (2, 9)
    for r in range(2):
        h = m.forward_packed(ids[r], torch.arange(10), torch.tensor([0, 10]), 10)
        ref = torch.log_softmax(m.logits(h).float(), -1)[:-1].gather(-1, ids[r, 1:, None]).squeeze(-1)
        assert (lp[r] - ref).abs().max().item() < 1e-3


def test_hf_greedy_generation_follows_native_argmax():
    from lumenrl_b200.engine.inference.hf_engine import HFEngine
    m = _native()
    eng = HFEngine.from_native(m)
    prompt = torch.randint(0, m.args.vocab_size, (1, 6), generator=torch.Generator().manual_seed(1))
    seqs, mask = eng.generate(prompt, max_new_tokens=4, do_sample=False)
    assert seqs.shape == (1, 10) and bool(mask.all())
    cur = prompt[0]
    for _ in range(4):
        T = cur.shape[0]
        h = m.forward_packed(cur, torch.arange(T), torch.tensor([0, T]), T)
        nxt = m.logits(h)[-1].argmax()
        cur = torch.cat([cur, nxt.view(1)])
    assert torch.equal(seqs[0], cur)


def test_hf_update_weights_checks_coverage():
    from lumenrl_b200.engine.inference.hf_engine import HFEngine
    m = _native()
    eng = HFEngine.from_native(m)
    sd = {k: v.detach().clone() for k, v in m.hf_state_dict().items()}
    assert eng.update_weights(sd) == len(sd)
    partial = dict(sd)
    partial.pop(next(iter(partial)))
    with pytest.raises(KeyError, match="coverage"):
        eng.update_weights(partial)
    with pytest.raises(KeyError, match="coverage"):
        eng.update_weights({**sd, "model.layers.99.mlp.up_proj.weight": torch.zeros(1)})


def test_native_loader_rejects_unexpected_keys():
    m = _native()
    sd = {k: v.detach().clone() for k, v in m.hf_state_dict().items()}
    with pytest.raises(KeyError, match="unexpected"):
        m.load_hf_state_dict({**sd, "model.foo.weight": torch.zeros(2)}, strict=True)
    assert m.load_hf_state_dict(sd, strict=True) == []


def test_generation_interface_round_trip():
    from lumenrl_b200.core.protocol import DataProto
    from lumenrl_b200.engine.inference.hf_engine import GenerationInterface, HFEngine
    m = _native()
    gi = GenerationInterface(lambda: HFEngine.from_native(m))
    gi.prepare_for_generation()
    batch = DataProto(tensors={"input_ids": torch.randint(0, m.args.vocab_size, (3, 5))},
                      meta={"sampling_params": {"max_new_tokens": 3, "do_sample": False}})
    out = gi.generate(batch)
    assert out["sequences"].shape == (3, 8) and out.meta["sampling_params"]["max_new_tokens"] == 3
    gi.finish_generation(release=True)


def test_rollout_engine_vocab_limit_never_samples_oov():
    """Ids at or past the limit (padded vocabulary rows) are never drawn."""
    from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
    m = _native()
    with torch.no_grad():
        m.lm_head[1000:] += 50.0          # make the padded rows overwhelmingly likely
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=64, use_cuda_graph=False, vocab_limit=1000)
    out = eng.generate([[1, 2, 3, 4]], SamplingParams(max_new_tokens=6, n=2, seed=0, stop_at_eos=False))
    assert int(out.responses.max()) < 1000


def _native_moe():
    from lumenrl_b200.models.config import tiny_qwen3_moe
    from lumenrl_b200.models.qwen3 import Qwen3Model
    m = Qwen3Model(tiny_qwen3_moe(), dtype=torch.float32, requires_grad=False)
    m.init_weights(3)
    return m


def test_hf_moe_twin_routes_experts_into_fused_parameters():
    """transformers' Qwen3-MoE module keeps fused [E, 2F, H] / [E, H, F]
    expert parameters; the per-expert export is fused on the way in and the
    twin scores like the native model."""
    from lumenrl_b200.engine.inference.hf_engine import HFEngine
    m = _native_moe()
    eng = HFEngine.from_native(m)
    ids = torch.randint(0, m.args.vocab_size, (2, 10), generator=torch.Generator().manual_seed(1))
    lp = eng.compute_log_probs(ids)
    for r in range(2):
        h = m.forward_packed(ids[r], torch.arange(10), torch.tensor([0, 10]), 10)
        ref = torch.log_softmax(m.logits(h).float(), -1)[:-1].gather(-1, ids[r, 1:, None]).squeeze(-1)
        assert (lp[r] - ref).abs().max().item() < 1e-4


def test_expert_spellings_round_trip_and_native_loader_takes_both():
    from lumenrl_b200.sync.moe_weights import fuse_experts, route_expert_weights, split_experts
    m = _native_moe()
    per = m.hf_state_dict()
    fused = m.hf_state_dict(fused_experts=True)
    assert any(k.endswith("experts.gate_up_proj") for k in fused)
    f2 = fuse_experts(per)
    assert f2.keys() == fused.keys() and all(torch.equal(f2[k], fused[k]) for k in fused)
    p2 = split_experts(fused)
    assert p2.keys() == per.keys() and all(torch.equal(p2[k], per[k]) for k in per)
    assert route_expert_weights(per, fused.keys()).keys() == fused.keys()
    assert route_expert_weights(fused, per.keys()).keys() == per.keys()
    # the native loader accepts the fused spelling (strict coverage still holds)
    m2 = _native_moe()
    m2.init_weights(11)
    m2.load_hf_state_dict({k: v.clone() for k, v in fused.items()})
    assert torch.equal(m2.flat, m.flat)


def test_fusing_rejects_a_missing_expert():
    from lumenrl_b200.sync.moe_weights import fuse_experts
    per = _native_moe().hf_state_dict()
    gone = next(k for k in per if ".experts.1.up_proj" in k)
    with pytest.raises(KeyError):
        fuse_experts({k: v for k, v in per.items() if k != gone})
