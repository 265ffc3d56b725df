"""Rollout engine on the GPU: the CUDA-graph decode step (paged attention,
fused QK-norm+RoPE+KV write, sampler) must reproduce the training forward's
log-probs under teacher forcing, with and without shared-prefix attention."""

import pytest
import torch

from lumenrl_b200 import ops
from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
from lumenrl_b200.models.config import tiny_qwen3
from lumenrl_b200.models.qwen3 import Qwen3Model

pytestmark = pytest.mark.gpu


def _model(dev, layers=2):
    m = Qwen3Model(tiny_qwen3(layers=layers), device=dev, dtype=torch.bfloat16, requires_grad=False)
    m.init_weights(0)
    return m


def _teacher_forced(m, prompt, resp):
    seq = list(prompt) + list(resp)
    dev = m.flat.device
    ids = torch.tensor(seq, device=dev)
    h = m.forward_packed(ids, torch.arange(len(seq), device=dev),
                         torch.tensor([0, len(seq)], device=dev, dtype=torch.int32), len(seq))
    lp, _ = ops.token_logprob(h[:-1], m.lm_head, ids[1:])
    return lp[len(prompt) - 1:].float()


@pytest.mark.parametrize("shared", [True, False])
def test_graph_decode_logprobs_match_training_forward(cuda, shared):
    m = _model(cuda)
    eng = RolloutEngine(m, max_num_seqs=16, max_model_len=256, block_size=16, use_cuda_graph=True,
                        shared_prefix_attention=shared)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(3, 2048, (L,), generator=g).tolist() for L in (40, 70)]
    out = eng.generate(prompts, SamplingParams(max_new_tokens=48, n=8, seed=5, eos_token_id=None))
    assert out.responses.shape == (16, 48)
    worst = 0.0
    with torch.no_grad():
        for r in range(16):
            ref_lp = _teacher_forced(m, prompts[r // 8], out.responses[r].tolist())
            worst = max(worst, (ref_lp - out.logprobs[r]).abs().max().item())
    # bf16 weights and activations on both sides; only the kernel order differs
    assert worst < 0.15, worst
    assert eng.cache.allocator.num_free == eng.cache.num_blocks - 1


def test_shared_and_plain_decode_agree(cuda):
    """Same seeds and weights: the shared-prefix decode graph samples the same
    first tokens, and near-identical log-probs, as the per-row graph."""
    m = _model(cuda)
    g = torch.Generator().manual_seed(2)
    prompts = torch.randint(3, 2048, (2, 64), generator=g)
    outs = []
    for shared in (True, False):
        eng = RolloutEngine(m, max_num_seqs=16, max_model_len=256, block_size=16, use_cuda_graph=True,
                            shared_prefix_attention=shared)
        outs.append(eng.generate(prompts.to(cuda), SamplingParams(max_new_tokens=8, n=8, seed=9, eos_token_id=None)))
    a, b = outs
    assert torch.equal(a.responses[:, :2], b.responses[:, :2])
    same = (a.responses == b.responses).all(1)
    assert (a.logprobs[same] - b.logprobs[same]).abs().max().item() < 0.05


def test_fp8_rollout_graph_decode(cuda):
    """W8A8 blockwise rollout (tcgen05 FP8 GEMM) inside the CUDA-graph decode
    step stays close to the bf16 training forward."""
    from lumenrl_b200.quant.fp8 import FP8Config
    m = _model(cuda)
    eng = RolloutEngine(m, max_num_seqs=16, max_model_len=256, block_size=16, use_cuda_graph=True,
                        fp8_rollout=FP8Config(precision="fp8"))
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(3, 2048, (64,), generator=g).tolist()]
    out = eng.generate(prompts, SamplingParams(max_new_tokens=32, n=8, seed=7, eos_token_id=None))
    with torch.no_grad():
        diffs = [(_teacher_forced(m, prompts[0], out.responses[r].tolist()) - out.logprobs[r]).abs().mean().item()
                 for r in range(8)]
    assert max(diffs) < 0.1, diffs
    assert ops.fp8_gemm_status() == 0


def test_moe_graph_decode_matches_eager_with_routes(cuda):
    """MoE rollout: the decode step is captured in a CUDA graph (device routing,
    grouped tcgen05 expert GEMMs) and reproduces eager decoding: the same
    samples, log-probs and recorded expert ids (rollout routing replay), over
    two generate() calls that reuse the captured graph."""
    from lumenrl_b200.models.config import tiny_qwen3_moe
    m = Qwen3Model(tiny_qwen3_moe(), device=cuda, dtype=torch.bfloat16, requires_grad=False)
    m.init_weights(0)
    sp = SamplingParams(max_new_tokens=12, n=2, seed=4, stop_at_eos=False)
    prompts = [[3 + i for i in range(20)], [7 + i for i in range(9)]]
    graph = RolloutEngine(m, max_num_seqs=8, max_model_len=64, block_size=16, use_cuda_graph=True)
    eager = RolloutEngine(m, max_num_seqs=8, max_model_len=64, block_size=16, use_cuda_graph=False)
    assert graph.use_cuda_graph
    for call in range(2):
        a = graph.generate(prompts, sp)
        b = eager.generate(prompts, sp)
        assert torch.equal(a.responses, b.responses), call
        assert (a.logprobs - b.logprobs).abs().max().item() < 1e-3
        assert len(a.routed_experts) == len(b.routed_experts) == 4
        for ra, rb in zip(a.routed_experts, b.routed_experts):
            assert torch.equal(ra, rb), call
