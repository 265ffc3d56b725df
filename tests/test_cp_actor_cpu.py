"""Context parallelism in the training engine on 2 gloo CPU ranks: the ranks
of one CP group split every sequence into zigzag chunks and run attention as a
ring; the scored log-probs and one GRPO update equal the single-process ones."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batch(seed: int = 0):
    from lumenrl_b200.core.protocol import DataProto
    g = torch.Generator().manual_seed(seed)
    B, P, R = 4, 12, 9
    plen = torch.tensor([12, 7, 10, 5])
    rlen = torch.tensor([9, 4, 7, 9])
    mask = (torch.arange(R).unsqueeze(0) < rlen.unsqueeze(1)).float()
    return DataProto({"prompt_ids": torch.randint(3, 2048, (B, P), generator=g), "prompt_lengths": plen,
                      "responses": torch.randint(3, 2048, (B, R), generator=g), "response_lengths": rlen,
                      "response_mask": mask, "old_log_probs": -torch.rand(B, R, generator=g) * 8,
                      "advantages": torch.randn(B, generator=g)})


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lumenrl_b200.core.config import GRPOConfig
        from lumenrl_b200.engine.training.actor import ActorEngine
        from lumenrl_b200.models.config import tiny_llama
        from lumenrl_b200.parallel.context_parallel import make_dp_cp_groups
        from lumenrl_b200.parallel.dist import ParallelState
        g = make_dp_cp_groups(2)
        st = ParallelState(world_size=world, rank=rank, cp_size=2, cp_rank=rank, cp_group=g)
        cp_eng = ActorEngine(tiny_llama(), st, lr=1e-3, seed=3)
        ref_eng = ActorEngine(tiny_llama(), ParallelState(), lr=1e-3, seed=3)
        b = _batch()
        lp_cp, ent_cp = cp_eng.compute_log_probs(b)
        lp_ref, ent_ref = ref_eng.compute_log_probs(b)
        m = b.tensors["response_mask"] > 0
        err_lp = float((lp_cp - lp_ref)[m].abs().max())
        err_ent = float((ent_cp - ent_ref)[m].abs().max())
        cfg = GRPOConfig()
        g_cp = cp_eng.update_policy(b, cfg, "grpo", rows_per_micro=2)["actor/grad_norm"]
        g_ref = ref_eng.update_policy(b, cfg, "grpo", rows_per_micro=2)["actor/grad_norm"]
        n = cp_eng.model.layout.numel
        dw = float((cp_eng.model.flat[:n] - ref_eng.model.flat[:n]).abs().max())
        moved = float((ref_eng.model.flat[:n] - ActorEngine(tiny_llama(), ParallelState(), seed=3,
                                                            trainable=False).model.flat[:n]).abs().max())
        q.put((rank, {"lp": err_lp, "ent": err_ent, "dw": dw, "moved": moved, "gn": abs(g_cp - g_ref) / g_ref,
                      "g_cp": g_cp, "g_ref": g_ref}))
    except Exception as e:  # surfaced by the parent
        import traceback
        q.put((rank, {"error": traceback.format_exc()[-2000:] + repr(e)}))
    dist.destroy_process_group()


def test_cp2_actor_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29720 + os.getpid() % 100
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, r in res:
        assert "error" not in r, r
        assert r["lp"] < 1e-4 and r["ent"] < 1e-4, (rank, r)
        assert r["gn"] < 1e-4, (rank, r["g_cp"], r["g_ref"])   # same global gradient norm
        assert r["moved"] > 1e-4, r                  # the update did something
        # Adam's first step is ~lr * sign(g): weights whose gradient is at the
        # rounding level may differ by a fraction of one step, no more
        assert r["dw"] < 0.1 * r["moved"], (rank, r)
