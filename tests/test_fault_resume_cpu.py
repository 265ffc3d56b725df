"""Host-side fault injection and checkpoint resume on 2 gloo CPU ranks
(reference: crash recovery is checkpoint-resume, ``rl_trainer.py:1235-1376``;
``callbacks.py:55-186``).

Run A trains 4 GRPO steps without interruption.  Run B checkpoints every 2
steps, and rank 1 raises in the middle of step 3 (rollout done, policy update
not started) and exits; rank 0's next collective with the dead rank must end
in an error within the short process-group timeout, not hang.  Run C
restarts both ranks on the same checkpoint directory: it resumes after step 2
and trains steps 3-4.  Its weights and its step-3/4 rewards equal run A's."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class InjectedFault(RuntimeError):
    pass


def _leave(q, item):
    q.put(item)
    q.close()
    q.join_thread()                      # the item is in the pipe before the process vanishes
    os._exit(0)


def _worker(rank, world, port, mode, root, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import tiny_llama
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.trainer.callbacks import CheckpointCallback
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec, RLTrainer

    st = init_distributed(backend="gloo", timeout_s=20.0, device="cpu")
    cfg = LumenRLConfig.from_yaml(os.path.join(HERE, "configs", "grpo_tiny_cpu.yaml"),
                                  ["num_training_steps=4", "algorithm.grpo.num_generations=4"])
    spec = RLRunSpec(prompts_per_step=4, prompt_len=16, max_new_tokens=16, reward="contains_token",
                     eos_token_id=None)
    tr = RLTrainer(cfg, tiny_llama(), spec, st).setup()
    if mode != "plain":
        tr.callbacks = [CheckpointCallback(root, save_steps=2, save_total_limit=3)]
    if mode == "crash" and rank == 1:
        real_update = tr.actor.update_policy

        def update_then_die(*a, **k):
            if tr.global_step == 2:      # the third step: its rollout ran, its update has not
                raise InjectedFault("rank 1 dies in the middle of step 3")
            return real_update(*a, **k)
        tr.actor.update_policy = update_then_die
    try:
        hist = tr.train()
        out = ("ok", [m["step"] for m in hist], [float(m["reward/mean"]) for m in hist],
               tr.actor.model.flat.clone().numpy())
    except InjectedFault as e:
        _leave(q, (rank, ("injected", str(e))))   # no goodbye to the group, like a crashed rank
    except Exception as e:               # rank 0: the collective with the dead rank failed
        _leave(q, (rank, ("error", type(e).__name__)))
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def _run(mode, root, port):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, root, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


@pytest.mark.timeout(600)
def test_rank_failure_is_reported_and_training_resumes_from_checkpoint(tmp_path):
    base = 29100 + os.getpid() % 300
    plain = _run("plain", str(tmp_path / "unused"), base)
    assert plain[0][0] == "ok" and plain[0][1] == [1, 2, 3, 4]

    root = str(tmp_path / "ck")
    crashed = _run("crash", root, base + 1)
    assert crashed[1][0] == "injected"
    assert crashed[0][0] == "error"              # rank 0 got an exception, not a hang
    from lumenrl_b200.utils.checkpoint import latest_step
    assert latest_step(root) == 2                # the last complete checkpoint

    resumed = _run("resume", root, base + 2)
    for r in (0, 1):
        assert resumed[r][0] == "ok"
        assert resumed[r][1] == [3, 4]           # picked up after step 2
    assert resumed[0][2] == plain[0][2][2:]      # same rollouts and rewards as the uninterrupted run
    assert (resumed[0][3] == plain[0][3]).all()  # and the same weights
    assert (resumed[1][3] == plain[1][3]).all()
