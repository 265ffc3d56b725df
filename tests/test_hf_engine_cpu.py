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
