"""CPU tier for the remaining components: checkpoints + HF export, the
assembler, seqlen balancing, async queue, weight sync, Eagle3, OPD, SFT."""

import os

import pytest
import torch

from lumenrl_b200.core.config import LumenRLConfig
from lumenrl_b200.core.protocol import DataProto
from lumenrl_b200.models.config import tiny_llama, tiny_qwen3
from lumenrl_b200.parallel.dist import ParallelState

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_checkpoint_roundtrip_and_hf_export(tmp_path):
    from lumenrl_b200.engine.training.actor import ActorEngine
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.utils.checkpoint import CheckpointManager, load_hf_safetensors, save_hf_safetensors
    e = ActorEngine(tiny_qwen3(), ParallelState(), lr=1e-2, seed=3)
    e.opt.grad.normal_()
    e.opt.step()
    mgr = CheckpointManager(str(tmp_path / "ck"), save_total_limit=2)
    for s in (1, 2, 3):
        mgr.save(e, s)
    assert mgr.steps() == [2, 3]
    e2 = ActorEngine(tiny_qwen3(), ParallelState(), lr=1e-2, seed=9)
    assert mgr.load_latest(e2) == 3
    assert torch.equal(e2.opt.master, e.opt.master) and torch.equal(e2.model.flat, e.model.flat)
    files = save_hf_safetensors(e.model, str(tmp_path / "hf"), dtype=torch.float32)
    assert files and os.path.isfile(tmp_path / "hf" / "model.safetensors.index.json")
    m3 = Qwen3Model(tiny_qwen3(), dtype=torch.float32)
    load_hf_safetensors(m3, str(tmp_path / "hf"))
    assert torch.equal(m3.flat[: e.model.layout.numel], e.model.flat[: e.model.layout.numel])


def test_checkpoint_crash_keeps_previous_step_and_restores_cursor(tmp_path, monkeypatch):
    """A save that dies half way leaves no half-written file under its final
    name and the tracker still names the last complete step; resume restores
    the data cursor."""
    from lumenrl_b200.engine.training.actor import ActorEngine
    from lumenrl_b200.utils import checkpoint as ck

    class Cursor:
        def __init__(self, pos=0):
            self.pos = pos

        def state_dict(self):
            return {"pos": self.pos}

        def load_state_dict(self, sd):
            self.pos = sd["pos"]

    e = ActorEngine(tiny_qwen3(), ParallelState(), lr=1e-2, seed=3)
    root = str(tmp_path / "ck")
    ck.save_sharded(e, root, 1, 0, 1, {"data": Cursor(7).state_dict()})
    real_save = torch.save

    def dying_save(obj, path, *a, **k):
        if "extra_state" in str(path):
            with open(path, "wb") as f:
                f.write(b"partial")
            raise OSError("disk went away")
        return real_save(obj, path, *a, **k)
    monkeypatch.setattr(torch, "save", dying_save)
    with pytest.raises(OSError):
        ck.save_sharded(e, root, 2, 0, 1, {"data": Cursor(9).state_dict()})
    monkeypatch.setattr(torch, "save", real_save)
    assert ck.latest_step(root) == 1
    d2 = os.path.join(root, "global_step_2", "actor")
    assert not os.path.exists(os.path.join(d2, "extra_state_world_size_1_rank_0.pt"))
    cur = Cursor(0)
    e2 = ActorEngine(tiny_qwen3(), ParallelState(), lr=1e-2, seed=9)
    assert ck.load_sharded(e2, root, 0, 1, data=cur) == 1
    assert cur.pos == 7


def test_hf_export_loads_in_transformers(tmp_path):
    transformers = pytest.importorskip("transformers")
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.utils.checkpoint import save_hf_safetensors
    m = Qwen3Model(tiny_qwen3(), dtype=torch.float32, requires_grad=False)
    m.init_weights(1)
    save_hf_safetensors(m, str(tmp_path / "hf"), dtype=torch.float32)
    hf = transformers.AutoModelForCausalLM.from_pretrained(str(tmp_path / "hf"), torch_dtype=torch.float32)
    ids = torch.randint(0, 2048, (1, 12))
    ref_logits = hf(ids).logits[0]
    h = m.forward_packed(ids[0], torch.arange(12), torch.tensor([0, 12]), 12)
    ours = m.logits(h)
    assert (ours - ref_logits).abs().max().item() < 1e-3


def test_assembler_and_policy():
    from lumenrl_b200.architecture.assembly import RuntimeAssembler
    cfg = LumenRLConfig()
    g = RuntimeAssembler(cfg).build_graph()
    assert g["trainer_cls"].__name__ == "RLTrainer"
    cfg.algorithm.name = "opd"
    assert RuntimeAssembler(cfg).build_graph()["trainer_cls"].__name__ == "OPDTrainer"
    cfg.algorithm.name = "grpo"
    cfg.async_training.enabled = True
    assert RuntimeAssembler(cfg).build_graph()["trainer_cls"].__name__ == "AsyncRLTrainer"
    cfg.assembly.training_backend = "deepspeed"
    with pytest.raises(ValueError):
        RuntimeAssembler(cfg).build_graph()


def test_seqlen_balancing():
    from lumenrl_b200.utils.seqlen_balancing import karmarkar_karp, partition_stats, seq_cost
    lens = [1000, 900, 800, 100, 90, 80, 70, 60]
    parts = karmarkar_karp([seq_cost(l) for l in lens], 2)
    assert sorted(i for p in parts for i in p) == list(range(8)) and all(len(p) == 4 for p in parts)
    assert partition_stats(lens, parts)["balance/imbalance"] < 1.5   # optimum for this set is 1.44


def test_async_queue_staleness():
    from lumenrl_b200.trainer.async_trainer import AsyncMessageQueue, SampleItem
    q = AsyncMessageQueue(maxsize=10, staleness_threshold=0.5)
    for v in (0, 0, 1, 1):
        q.put(SampleItem(DataProto({"x": torch.zeros(1)}), v))
    q.current_param_version = 1
    got = q.get_batch(2, timeout=2)
    assert [g.param_version for g in got] == [0, 1]     # one stale allowed (0.5 * 2), the other dropped
    assert q.dropped == 1


def test_filesystem_weight_sync(tmp_path):
    from lumenrl_b200.sync.weight_sync import FilesystemWeightSync
    s = FilesystemWeightSync(str(tmp_path), keep_versions=2)
    for _ in range(3):
        s.push({"w": torch.ones(3)})
    sd, ver = s.pull()
    assert ver == 3 and torch.equal(sd["w"], torch.ones(3))
    assert not (tmp_path / "v1").exists()


def test_eagle3_tiny_forward_backward():
    from lumenrl_b200.models.eagle3 import Eagle3Model, cached_tree_attention
    torch.manual_seed(0)
    H, V, Vd = 64, 300, 100
    m = Eagle3Model(H, V, Vd, num_heads=4, num_kv_heads=2, head_dim=16, ffn=128, length=3)
    T = 20
    ids = torch.randint(0, V, (T,))
    cu = torch.tensor([0, 12, 20])
    out = m(ids, torch.randn(T, 3 * H), torch.randn(T, H), torch.randn(V, H), torch.randn(V, H), cu,
            torch.ones(T))
    out["loss"].backward()
    assert len(out["losses"]) == 3 and m.fc.weight.grad is not None
    # tree attention with only step-0 keys equals plain causal attention
    from lumenrl_b200.ops.reference import attention_varlen
    q, k, v = torch.randn(T, 4, 16), torch.randn(T, 2, 16), torch.randn(T, 2, 16)
    a = cached_tree_attention(q, [(k, v)], cu, 0.25)
    b = attention_varlen(q, k, v, cu, True, 0.25)
    assert torch.allclose(a, b, atol=1e-5)


def test_spec_distill_and_sft_and_opd_steps():
    from lumenrl_b200.trainer.opd_trainer import OPDTrainer
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec
    from lumenrl_b200.trainer.sft_trainer import SFTTrainer
    from lumenrl_b200.trainer.spec_distill_trainer import SpecDistillSpec, SpecDistillTrainer
    st = ParallelState()
    sd = SpecDistillTrainer(tiny_qwen3(layers=4), SpecDistillSpec(aux_layers=(0, 1, 2), draft_vocab=256, ttt_length=2,
                                                                 seq_len=16, batch_per_rank=2, draft_heads=4,
                                                                 draft_kv_heads=2, draft_ffn=128), st)
    r = sd.step()
    assert r["loss"] > 0 and len(r["acc"]) == 2
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"))
    sft = SFTTrainer(cfg, tiny_llama(), st)
    b = DataProto({"prompt_ids": torch.randint(3, 2048, (4, 8)), "prompt_lengths": torch.full((4,), 8),
                   "responses": torch.randint(3, 2048, (4, 6)), "response_lengths": torch.tensor([6, 5, 4, 6]),
                   "response_mask": (torch.arange(6).unsqueeze(0) < torch.tensor([6, 5, 4, 6]).unsqueeze(1)).float()})
    l1 = sft.step(b)["sft/loss"]
    assert l1 > 0
    cfg.algorithm.name = "opd"
    opd = OPDTrainer(cfg, tiny_llama(), RLRunSpec(prompts_per_step=2, prompt_len=8, max_new_tokens=6,
                                                  eos_token_id=None), st).setup()
    assert opd.step()["opd/kl"] > 0
