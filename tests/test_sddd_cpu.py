"""SDDD layout on CPU ranks (gloo): three teacher ranks stream hidden states
through the ring to one draft rank; after two steps the draft equals a
single-process trainer that ran the same three teacher batches per step."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import dataclasses

from lumenrl_b200.models.config import tiny_qwen3
from lumenrl_b200.parallel.dist import ParallelState
from lumenrl_b200.trainer.spec_distill_trainer import SDDDTrainer, SpecDistillSpec, SpecDistillTrainer

TEACHER = dataclasses.replace(tiny_qwen3(), num_layers=3)
SPEC = dict(aux_layers=(0, 1, 2), draft_vocab=256, ttt_length=3, seq_len=32, batch_per_rank=2, lr=1e-3,
            draft_heads=4, draft_kv_heads=2, draft_ffn=128)
STEPS = 2


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    tr = SDDDTrainer(TEACHER, SpecDistillSpec(**SPEC), ParallelState(rank=rank, world_size=world),
                     num_teacher=3, seed=5)
    outs = [tr.step() for _ in range(STEPS)]
    if not tr.is_teacher:
        q.put((rank, [o["loss"] for o in outs], {k: v.detach().clone() for k, v in tr.draft.state_dict().items()}))
    else:
        q.put((rank, None, None))
    dist.barrier()
    tr.close()
    dist.destroy_process_group()


def test_three_teachers_one_draft_match_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {r: (l, sd) for r, l, sd in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    losses, sd = res[3]
    torch.manual_seed(5)
    single = SpecDistillTrainer(TEACHER, SpecDistillSpec(**SPEC), ParallelState(), seed=5)
    ref_losses = []
    for s in range(STEPS):
        batches = []
        for t in range(3):
            ids = single._ids(s, t)
            cu = torch.arange(0, ids.numel() + 1, SPEC["seq_len"], dtype=torch.int32)
            aux, last = single.teacher_forward(ids, cu)
            batches.append((ids, aux, last))
        ref_losses.append(single.draft_update(batches)["loss"])
    for a, b in zip(losses, ref_losses):
        assert abs(a - b) <= 1e-5 * max(1.0, abs(b)), (losses, ref_losses)
    for k, v in single.draft.state_dict().items():
        assert torch.allclose(sd[k], v, atol=1e-6), k
