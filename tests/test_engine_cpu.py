"""Native rollout engine on CPU: log-prob consistency with the training
forward, prefix sharing, R3 routes, sleep/wake, sampling determinism."""

import torch

from lumenrl_b200 import ops
from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
from lumenrl_b200.engine.training.packing import make_micro_batches, pack_rows
from lumenrl_b200.models.config import tiny_llama, tiny_qwen3_moe
from lumenrl_b200.models.qwen3 import Qwen3Model


def _model(args):
    m = Qwen3Model(args, dtype=torch.float32, requires_grad=False)
    m.init_weights(0)
    return m


def test_rollout_logprobs_match_teacher_forcing():
    m = _model(tiny_llama())
    eng = RolloutEngine(m, max_num_seqs=8, max_model_len=64, block_size=16, use_cuda_graph=False)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(3, 2048, (L,), generator=g).tolist() for L in (20, 16)]
    out = eng.generate(prompts, SamplingParams(max_new_tokens=12, n=3, seed=3, eos_token_id=None))
    assert out.responses.shape == (6, 12)
    for r in range(6):
        p = prompts[r // 3]
        seq = p + out.responses[r].tolist()
        ids = torch.tensor(seq)
        h = m.forward_packed(ids, torch.arange(len(seq)), torch.tensor([0, len(seq)]), len(seq))
        lp, _ = ops.token_logprob(h[:-1], m.lm_head, ids[1:])
        assert (lp[len(p) - 1:] - out.logprobs[r]).abs().max() < 2e-3
    # all blocks returned to the pool
    assert eng.cache.allocator.num_free == eng.cache.num_blocks - 1


def test_seed_determinism_and_sleep_wake():
    m = _model(tiny_llama())
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=48, block_size=16, use_cuda_graph=False)
    prompts = [[5, 6, 7, 8, 9]]
    a = eng.generate(prompts, SamplingParams(max_new_tokens=8, n=4, seed=11, eos_token_id=None))
    eng.sleep()
    assert not eng.cache.awake
    b = eng.generate(prompts, SamplingParams(max_new_tokens=8, n=4, seed=11, eos_token_id=None))
    assert torch.equal(a.responses, b.responses)
    c = eng.generate(prompts, SamplingParams(max_new_tokens=8, n=4, seed=12, eos_token_id=None))
    assert not torch.equal(a.responses, c.responses)
    # decode graphs survive a sleep/wake that returns the same KV block, and are
    # dropped when the pool moves
    assert eng._graphs
    before = eng.cache.pool_ptr
    eng.sleep()
    eng.wake()
    assert bool(eng._graphs) == (eng.cache.pool_ptr == before)
    eng.sleep()
    eng._graphs_pool_ptr = -1
    eng.wake()
    assert not eng._graphs and eng._graphs_pool_ptr == eng.cache.pool_ptr
    d = eng.generate(prompts, SamplingParams(max_new_tokens=8, n=4, seed=11, eos_token_id=None))
    assert torch.equal(a.responses, d.responses)


def test_eos_and_waves():
    m = _model(tiny_llama())
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=40, block_size=16, use_cuda_graph=False)
    prompts = [[3, 4, 5]] * 3
    out = eng.generate(prompts, SamplingParams(max_new_tokens=10, n=2, seed=0, eos_token_id=None))
    assert out.responses.shape[0] == 6 and out.prompt_index.tolist() == [0, 0, 1, 1, 2, 2]
    # force EOS: every token id is EOS when the vocab is tiny
    tok = out.responses[0, 0].item()
    out2 = eng.generate([[3, 4, 5]], SamplingParams(max_new_tokens=10, n=2, seed=0, eos_token_id=tok))
    assert out2.response_lengths[0].item() == 1


def test_moe_routes_recorded():
    m = _model(tiny_qwen3_moe())
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=40, block_size=16, use_cuda_graph=False)
    out = eng.generate([[3, 4, 5, 6]], SamplingParams(max_new_tokens=6, n=2, seed=0, eos_token_id=None))
    r = out.routed_experts[0]
    assert r.shape == (4 + 6 - 1, 2, 2)


def test_packing_and_micro_batches():
    pb = pack_rows([torch.tensor([1, 2, 3]), torch.tensor([4, 5])], [torch.tensor([7, 8]), torch.tensor([9])], "cpu")
    assert pb.input_ids.tolist() == [1, 2, 3, 7, 8, 4, 5, 9]
    assert pb.cu_seqlens.tolist() == [0, 5, 8]
    assert pb.score_index.tolist() == [2, 3, 6] and pb.targets.tolist() == [7, 8, 9]
    grid = pb.scatter(torch.tensor([0.1, 0.2, 0.3]), 2)
    assert torch.allclose(grid, torch.tensor([[0.1, 0.2], [0.3, 0.0]]))
    bins = make_micro_batches([10, 8, 6, 4, 2], token_budget=12)
    assert sorted(i for b in bins for i in b) == [0, 1, 2, 3, 4]
    assert all(sum([10, 8, 6, 4, 2][i] for i in b) <= 12 or len(b) == 1 for b in bins)


def test_shared_prefix_group_and_fallback():
    assert ops.shared_prefix_group(8, 4) == 8
    assert ops.shared_prefix_group(32, 4) == 16
    assert ops.shared_prefix_group(6, 16) == 3
    assert ops.shared_prefix_group(5, 16) == 1
    # the CPU path of the shared-prefix call is plain paged attention
    torch.manual_seed(0)
    B, Hq, Hk, D, bs = 4, 4, 2, 16, 8
    kc, vc = torch.randn(9, bs, Hk, D), torch.randn(9, bs, Hk, D)
    bt = torch.tensor([[1, 2, 3, 4], [1, 2, 5, 6], [1, 2, 7, 8], [1, 2, 3, 4]], dtype=torch.int32)
    lens = torch.tensor([20, 25, 17, 32], dtype=torch.int32)
    q = torch.randn(B, Hq, D)
    a = ops.paged_decode_attention_shared(q, kc, vc, bt, lens, torch.full((B,), 16, dtype=torch.int32), 2, 0.25)
    b = ops.paged_decode_attention(q, kc, vc, bt, lens, 0.25)
    assert torch.allclose(a, b)


def test_fp8_rollout_close_to_bf16_and_requantised_on_sync():
    """W8A8 blockwise rollout: log-probs stay close to the full-precision
    training forward, and a weight update re-quantises the rollout weights."""
    from lumenrl_b200.quant.fp8 import FP8Config
    m = _model(tiny_llama())
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=64, block_size=16, use_cuda_graph=False,
                        fp8_rollout=FP8Config(precision="fp8"))
    assert len(eng.runner.fp8.weights) == 4 * m.args.num_layers
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12]]
    out = eng.generate(prompts, SamplingParams(max_new_tokens=10, n=2, seed=3, eos_token_id=None))
    diffs = []
    for r in range(2):
        seq = prompts[0] + out.responses[r].tolist()
        ids = torch.tensor(seq)
        h = m.forward_packed(ids, torch.arange(len(seq)), torch.tensor([0, len(seq)]), len(seq))
        lp, _ = ops.token_logprob(h[:-1], m.lm_head, ids[1:])
        diffs.append((lp[len(prompts[0]) - 1:] - out.logprobs[r]).abs().mean())
    assert max(diffs) < 0.05, diffs
    name = "layers.0.wqkv"
    before, before_s = (t.clone() for t in eng.runner.fp8.weights[name])
    with torch.no_grad():
        m.p(name).mul_(2.0)
    eng.update_weights()
    after_q, after_s = eng.runner.fp8.weights[name]
    assert torch.equal(after_q.float(), before.float())   # same fp8 codes ...
    assert torch.allclose(after_s, 2 * before_s)          # ... and the scales follow the doubled weights


def test_continuous_batching_same_samples_fewer_steps():
    """More rows than slots: continuous batching refills finished slots with
    queued samples.  Every row equals the static-wave result for the same
    seed (per-row RNG counters), and fewer decode steps run."""
    eos = 2
    m = _model(tiny_llama())
    # make EOS likely (a few % per token): raise its logit along the final norm
    with torch.no_grad():
        m.lm_head[eos] = m.lm_head[eos] + 0.35 * m.p("norm").sign()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(3, 2048, (L,), generator=g).tolist() for L in (12, 16, 9, 20, 7, 14)]
    sp = SamplingParams(max_new_tokens=24, n=2, seed=7, eos_token_id=eos)

    def run(continuous: bool):
        eng = RolloutEngine(m, max_num_seqs=4, max_model_len=48, block_size=8, use_cuda_graph=False,
                            continuous_batching=continuous)
        out = eng.generate(prompts, sp)
        assert eng.cache.allocator.num_free == eng.cache.num_blocks - 1   # every block came back
        return out

    static, cont = run(False), run(True)
    assert torch.equal(static.response_lengths, cont.response_lengths)
    L = int(static.response_lengths.max())
    assert torch.equal(static.responses[:, :L], cont.responses[:, :L])
    assert (static.logprobs[:, :L] - cont.logprobs[:, :L]).abs().max() < 1e-5
    lens = static.response_lengths
    assert 1 <= int(lens.min()) < int(lens.max())          # rows really ended at different times
    st = cont.stats
    assert st["decode_steps"] < st["static_wave_decode_steps"]
    assert st["decode_steps_saved"] > 0
