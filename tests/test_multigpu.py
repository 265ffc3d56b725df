"""Multi-GPU: the fused NVLink optimizer step (peer-load reduce-scatter +
norm, clip + AdamW + bf16 peer-store broadcast) against the NCCL path, as
2 processes on 2 GPUs.  Skips with fewer than 2 GPUs."""

import datetime
import os
import random
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

# short process-group timeout: ranks that wait on a dead or stalled peer end in
# an error instead of holding the GPUs
_PG_TIMEOUT = datetime.timedelta(seconds=180)


def _need(world: int) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _worker(rank, world, port, q, nvls=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.engine.training.optimizer import ShardedFlatAdamW
    from lumenrl_b200.parallel.symm import NVLinkOptimizerComm
    n = 128 * world * 1000
    torch.manual_seed(0)
    w0 = torch.randn(n, device="cuda").to(torch.bfloat16)
    comm = NVLinkOptimizerComm(n, rank, world, nvls=nvls)
    comm.weights.tensor.copy_(w0)
    fused = ShardedFlatAdamW(comm.weights.tensor, world, rank, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1,
                             max_grad_norm=1.0, comm=comm)
    plain_w = w0.clone()
    plain = ShardedFlatAdamW(plain_w, world, rank, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)
    norms = []
    for step in range(3):
        g = torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 * step + rank))
        fused.grad.copy_(g)
        plain.grad.copy_(g)
        a = fused.step()
        b = plain.step()
        norms.append((a["grad_norm"], b["grad_norm"]))
    torch.cuda.synchronize()
    err = (comm.weights.tensor.float() - plain_w.float()).abs().max().item()
    q.put((rank, err, norms, comm.nvls))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("nvls", [True, False])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_optimizer_step_matches_nccl(world, nvls):
    """Fused step (nvls=True: NVLS multimem when the GPUs support it; False:
    peer loads and stores) against NCCL reduce-scatter + AdamW + all-gather."""
    _need(world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, world, port + (0 if nvls else 50), q, nvls))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    print("nvls path:", [r[3] for r in res])
    for rank, err, norms, _ in res:
        assert err <= 1e-2, (rank, err)
        for a, b in norms:
            assert abs(a - b) <= 1e-3 * max(1.0, b), (a, b)


def _allreduce_worker(rank, world, port, q, nvls):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.symm import NVLinkAllReduce
    from lumenrl_b200.trainer.spec_distill_trainer import allreduce_mean_grads
    comm = NVLinkAllReduce(4000, rank, world, nvls=nvls)          # small: buckets go through in pieces
    errs = []
    for step, (n, dt) in enumerate([(10003, torch.float32), (6001, torch.bfloat16), (8, torch.float32)]):
        g = torch.Generator(device="cuda").manual_seed(100 * step + rank)
        x = torch.randn(n, device="cuda", generator=g).to(dt)
        want = x.float().clone()
        dist.all_reduce(want)
        got = comm.all_reduce_(x.clone(), scale=1.0 / world).float()
        errs.append((got - want / world).abs().max().item())
    # the replicated-DP gradient path of the draft trainer
    lin = torch.nn.Linear(64, 48, device="cuda")
    lin.weight.grad = torch.full_like(lin.weight, float(rank + 1))
    lin.bias.grad = torch.full_like(lin.bias, float(2 * rank))
    allreduce_mean_grads(list(lin.parameters()), world, comm=comm)
    errs.append((lin.weight.grad - (world + 1) / 2).abs().max().item())
    errs.append((lin.bias.grad - (world - 1)).abs().max().item())
    comm.check()
    torch.cuda.synchronize()
    q.put((rank, errs, comm.nvls))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("nvls", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_nvlink_allreduce_matches_nccl(world, nvls):
    """Replicated-DP all-reduce on the peer-memory kernel (nvls=True: NVLS
    multimem when supported) against NCCL all_reduce, fp32 and bf16 buckets
    larger and smaller than the staging buffer."""
    _need(world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28700 + os.getpid() % 150 + (0 if nvls else 200)
    procs = [ctx.Process(target=_allreduce_worker, args=(r, world, port, q, nvls)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    print("nvls path:", [r[2] for r in res])
    for rank, errs, _ in res:
        assert errs[0] <= 1e-5 and errs[1] <= 2e-2 and errs[2] <= 1e-5, (rank, errs)
        assert errs[3] <= 1e-6 and errs[4] <= 1e-6, (rank, errs)


def _dead_peer_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.symm import CommTimeout, NVLinkOptimizerComm
    n = 128 * world * 64
    # plain peer loads / stores: no rank's memory is bound to an NVLS multicast object
    comm = NVLinkOptimizerComm(n, rank, world, wait_seconds=0.5, nvls=False)
    shard = n // world
    master = torch.zeros(shard, device="cuda")
    gs, m, v = torch.zeros_like(master), torch.zeros_like(master), torch.zeros_like(master)
    result = "no-error"
    if rank == 0:   # rank 1 "dies" before the step: it never enters the kernels
        try:
            comm.fused_step(0, shard, master, gs, m, v, 1e-3, (0.9, 0.95), 1e-8, 0.0, 1, 1.0, rendezvous=False)
        except CommTimeout:
            result = "timeout"
    torch.cuda.synchronize()
    q.put((rank, result))
    dist.barrier()           # both ranks leave between steps, nothing in flight
    comm.close()
    dist.destroy_process_group()


def test_dead_peer_becomes_comm_timeout():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + os.getpid() % 90
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "timeout"


def _ring_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.symm import CommTimeout
    from lumenrl_b200.transfer.p2p_ring import HiddenStateRing
    T, D = 2048, 4 * 1024   # one 16 MiB batch of bf16 hidden rows
    ring = HiddenStateRing(producer=0, consumer=1, slot_bytes=T * D * 2, nslots=2, wait_seconds=2.0)
    errs = []
    # randomised host delays before every launch skew the two ranks' kernels
    # against each other; the lap-numbered flags must still deliver every
    # batch intact and in order
    delay = random.Random(1234 + rank)
    for i in range(8):   # more batches than slots: the producer waits for released slots
        x = torch.randn(T, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(i)).to(torch.bfloat16)
        time.sleep(delay.uniform(0.0, 0.05))
        if rank == 0:
            ring.put(x)
        else:
            y = ring.get((T, D), torch.bfloat16)
            errs.append((y.float() - x.float()).abs().max().item())
            ring.release()
    torch.cuda.synchronize()
    ring.check()
    dist.barrier()
    # a batch the producer never pushes: the consumer's bounded wait expires
    timeout = "no-error"
    if rank == 1:
        ring.get((T, D), torch.bfloat16)
        torch.cuda.synchronize()
        try:
            ring.check()
        except CommTimeout:
            timeout = "timeout"
        ring._held = None
    q.put((rank, errs, timeout))
    dist.barrier()
    ring.close()
    dist.destroy_process_group()


def test_hidden_state_ring_nvlink():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29990 + os.getpid() % 9
    procs = [ctx.Process(target=_ring_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (e, t) for r, e, t in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    errs, timeout = res[1]
    assert len(errs) == 8 and max(errs) == 0.0
    assert timeout == "timeout"


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.tp_check import tp_layer_errors
    fused = tp_layer_errors("cuda", torch.bfloat16, fused=True, T=1024)
    plain = tp_layer_errors("cuda", torch.bfloat16, fused=False, T=1024)
    q.put((rank, fused, plain))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_fused_ag_rs_gemms(world):
    """TP + sequence parallel decoder layer, forward and backward, with the
    all-gather and reduce-scatter fused into tcgen05 GEMMs over NVLink; the
    result must match the unsharded bf16 layer about as closely as the NCCL
    path does."""
    _need(world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29980 + os.getpid() % 9 + world
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, fused, plain in res:
        assert fused["fused"] and not plain["fused"]
        for k in fused:
            if k == "fused":
                continue
            assert fused[k] < max(3 * plain[k], 2e-2), (rank, k, fused[k], plain[k])


def _cp_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.context_parallel import ring_attention, zigzag_indices
    S, H, Hk, D = 4096, 8, 2, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(1, h, S, D, device="cuda", generator=g).to(torch.bfloat16) for h in (H, Hk, Hk, H))
    idx = zigzag_indices(S, world, rank, "cuda")

    def rel(a, b):
        return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
    errs = {}
    # two calls with different inputs: the ring's receive slots are reused,
    # so stale contents would show up in the second
    for it, (sq, sv) in enumerate(((1.0, 1.0), (0.5, 2.0))):
        qi, vi = (q.float() * sq).to(q.dtype), (v.float() * sv).to(v.dtype)
        ql, kl, vl = (t[:, :, idx].clone().requires_grad_(True) for t in (qi, k, vi))
        o = ring_attention(ql, kl, vl)
        o.backward(do[:, :, idx])
        qf, kf, vf = (t.clone().requires_grad_(True) for t in (qi, k, vi))
        of = torch.nn.functional.scaled_dot_product_attention(qf, kf.repeat_interleave(H // Hk, 1),
                                                              vf.repeat_interleave(H // Hk, 1), is_causal=True)
        of.backward(do)
        for name, a, b in (("o", o, of[:, :, idx]), ("dq", ql.grad, qf.grad[:, :, idx]),
                           ("dk", kl.grad, kf.grad[:, :, idx]), ("dv", vl.grad, vf.grad[:, :, idx])):
            errs[name] = max(errs.get(name, 0.0), rel(a, b))
    out_q.put((rank, errs))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_ring_attention(world):
    """CP zigzag ring attention (flash blocks + LSE merge, K/V and dK/dV over
    the NVLink ring channel) against full causal attention, forward and
    backward, bf16, two calls."""
    _need(world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29970 + os.getpid() % 9 + world
    procs = [ctx.Process(target=_cp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs in res:
        for k, v in errs.items():
            assert v < 2e-2, (rank, k, v)


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.parallel.ep_check import ep_errors
    kw = dict(T=512, H=256, F=128, E=8, k=2)
    fused = ep_errors("cuda", torch.bfloat16, fused=True, **kw)
    plain = ep_errors("cuda", torch.bfloat16, fused=False, **kw)
    q.put((rank, fused, plain))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_nvlink_dispatch_combine(world):
    """EP MoE part: count exchange, dispatch and combine by peer stores,
    grouped tcgen05 expert GEMMs; forward and backward against all experts on
    one rank, as close as the NCCL all-to-all path."""
    _need(world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29960 + os.getpid() % 9 + world
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, fused, plain in res:
        assert fused["fused"] and not plain["fused"]
        for k in fused:
            if k != "fused":
                assert fused[k] < max(3 * plain[k], 3e-2), (rank, k, fused[k], plain[k])


def _p2p_sync_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.engine.inference.engine import RolloutEngine
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.models.qwen3 import Qwen3Model
    from lumenrl_b200.sync.weight_sync import P2PWeightSync
    m = Qwen3Model(tiny_qwen3(), device="cuda", dtype=torch.bfloat16, requires_grad=False)
    m.init_weights(rank)          # the two ranks start with different weights
    eng = RolloutEngine(m, max_num_seqs=4, max_model_len=64, block_size=16, use_cuda_graph=False) if rank == 1 else None
    sync = P2PWeightSync(m.flat.numel(), src=0, dst=1, engine=eng, bucket_size_mb=1)
    res = []
    for step in range(3):
        if rank == 0:
            with torch.no_grad():
                m.flat.add_(0.01)
            out = sync.sync(m.flat)
            dist.send(m.flat.contiguous(), 1)
        else:
            out = sync.sync()
            ref = torch.empty_like(eng.model.flat)
            dist.recv(ref, 0)
            bad = (eng.model.flat.view(torch.int16) != ref.view(torch.int16)).nonzero()
            if bad.numel():   # diagnose: which elements differ
                print(f"p2p sync step {step}: {bad.numel()} of {ref.numel()} elements differ, first {int(bad[0])}, "
                      f"last {int(bad[-1])}, flags {sync.sig.tensor[:8].tolist()}", flush=True)
            res.append(bad.numel() / ref.numel())
            # the engine generates from the synced weights
            g = eng.generate([[1, 2, 3]], __import__("lumenrl_b200.engine.inference.engine", fromlist=["x"])
                             .SamplingParams(max_new_tokens=4, n=2, seed=step))
            assert g.responses.shape == (2, 4)
        res.append(out["weight_sync/GBps"]) if rank == 0 else None
    q.put((rank, res))
    dist.barrier()
    sync.close()
    dist.destroy_process_group()


def test_p2p_weight_sync_to_separate_rollout_gpu():
    """Separated mode: the trainer GPU pushes its flat weights into the
    rollout GPU's buffer over NVLink; the rollout engine sees them at once."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29950 + os.getpid() % 9
    procs = [ctx.Process(target=_p2p_sync_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert len(res[1]) == 3 and max(res[1]) == 0.0, res[1]


def _sep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    from lumenrl_b200.core.config import LumenRLConfig
    from lumenrl_b200.models.config import tiny_qwen3_moe
    from lumenrl_b200.parallel.dist import ParallelState, init_distributed
    from lumenrl_b200.trainer.rl_trainer import RLRunSpec
    from lumenrl_b200.trainer.separated_trainer import SeparatedRLTrainer
    st = init_distributed()
    cfg = LumenRLConfig.from_dict({"algorithm": {"name": "grpo", "grpo": {"num_generations": 4}},
                                   "policy": {"learning_rate": 1e-5}, "num_training_steps": 2, "seed": 0})
    spec = RLRunSpec(prompts_per_step=4, prompt_len=64, max_new_tokens=32, reward="parity", eos_token_id=None)
    tr = SeparatedRLTrainer(cfg, tiny_qwen3_moe(), spec, st, num_rollout=1).setup()
    hist = [tr.step() for _ in range(2)]
    torch.cuda.synchronize()
    flat = tr.model.flat.clone()
    other = torch.empty_like(flat)
    if rank == 0:
        dist.send(flat, 1)
        q.put((rank, hist[-1].get("actor/grad_norm"), hist[-1].get("weight_sync/push_GBps"), None))
    else:
        dist.recv(other, 0)
        q.put((rank, None, hist[-1].get("weight_sync/push_GBps"), bool(torch.equal(other, flat))))
    dist.barrier()
    tr.close()
    dist.destroy_process_group()


def test_separated_trainer_and_rollout_gpus():
    """Separated mode on 2 GPUs: a tiny MoE GRPO step on the trainer GPU, the
    rollout on the other; the weights reach the rollout GPU by peer stores
    (P2PWeightSync) and equal the trainer's after every step."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29940 + os.getpid() % 9
    procs = [ctx.Process(target=_sep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (g, bw, same) for r, g, bw, same in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
    assert res[0][0] == res[0][0] and res[0][0] > 0      # finite, non-zero grad norm
    assert res[1][2] is True                             # rollout weights == trainer weights


def _sddd_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    import dataclasses
    from lumenrl_b200.models.config import tiny_qwen3
    from lumenrl_b200.parallel.dist import init_distributed
    from lumenrl_b200.trainer.spec_distill_trainer import SDDDTrainer, SpecDistillSpec
    st = init_distributed()
    spec = SpecDistillSpec(aux_layers=(0, 1, 2), draft_vocab=256, ttt_length=3, seq_len=128, batch_per_rank=2,
                           draft_heads=4, draft_kv_heads=2, draft_ffn=256)
    tr = SDDDTrainer(dataclasses.replace(tiny_qwen3(), num_layers=3), spec, st, num_teacher=world - 1, seed=3)
    outs = [tr.step() for _ in range(3)]
    torch.cuda.synchronize()
    tr.check()
    q.put((rank, [o.get("loss") for o in outs]))
    dist.barrier()
    tr.close()
    dist.destroy_process_group()


def test_sddd_teacher_streams_hidden_states_to_draft_gpu():
    """SDDD on 2 GPUs: the teacher GPU pushes ids + hidden states into the
    draft GPU's ring slots over NVLink; the draft trains on them."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29930 + os.getpid() % 9
    procs = [ctx.Process(target=_sddd_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    losses = res[1]
    assert len(losses) == 3 and all(l == l and l > 0 for l in losses)


def _cp_actor_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    try:
        from lumenrl_b200.core.protocol import DataProto
        from lumenrl_b200.engine.training.actor import ActorEngine
        from lumenrl_b200.models.config import tiny_qwen3
        from lumenrl_b200.parallel.context_parallel import make_dp_cp_groups
        from lumenrl_b200.parallel.dist import ParallelState
        dev = torch.device("cuda", rank)
        g = make_dp_cp_groups(world)
        st = ParallelState(world_size=world, rank=rank, local_rank=rank, device=dev, cp_size=world, cp_rank=rank,
                           cp_group=g)
        cp_eng = ActorEngine(tiny_qwen3(), st, seed=3, trainable=False)
        ref_eng = ActorEngine(tiny_qwen3(), ParallelState(device=dev), seed=3, trainable=False)
        gen = torch.Generator().manual_seed(0)
        B, P, R = 4, 300, 200
        plen, rlen = torch.tensor([300, 128, 257, 64]), torch.tensor([200, 77, 131, 200])
        b = DataProto({"prompt_ids": torch.randint(3, 2048, (B, P), generator=gen), "prompt_lengths": plen,
                       "responses": torch.randint(3, 2048, (B, R), generator=gen), "response_lengths": rlen,
                       "response_mask": (torch.arange(R).unsqueeze(0) < rlen.unsqueeze(1)).float()})
        lp_cp, _ = cp_eng.compute_log_probs(b, want_entropy=False)
        lp_ref, _ = ref_eng.compute_log_probs(b, want_entropy=False)
        m = b.tensors["response_mask"].to(dev) > 0
        q.put((rank, float((lp_cp - lp_ref)[m].abs().max())))
    except Exception as e:
        q.put((rank, repr(e)))
    dist.barrier()
    dist.destroy_process_group()


def test_context_parallel_actor_scoring_on_gpus():
    """The training engine with CP = 2 over two GPUs (zigzag shares, ring
    attention on the tcgen05 flash kernels, K/V over the NVLink ring) scores the
    same log-probs as one GPU with the whole sequences."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29890 + os.getpid() % 50
    procs = [ctx.Process(target=_cp_actor_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert isinstance(err, float), (rank, err)
        assert err < 5e-2, (rank, err)     # bf16 logits, log-prob difference in nats


def _sharded_engine_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    try:
        from lumenrl_b200.core.config import GRPOConfig
        from lumenrl_b200.core.protocol import DataProto
        from lumenrl_b200.engine.training.actor import ActorEngine
        from lumenrl_b200.engine.training.fsdp import ShardedParamActorEngine
        from lumenrl_b200.models.config import tiny_qwen3
        from lumenrl_b200.parallel.dist import ParallelState
        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(rank)
        B, P, R = 4, 40, 24
        rlen = torch.randint(8, R + 1, (B,), generator=g)
        b = DataProto({"prompt_ids": torch.randint(3, 2048, (B, P), generator=g), "prompt_lengths": torch.full((B,), P),
                       "responses": torch.randint(3, 2048, (B, R), generator=g), "response_lengths": rlen,
                       "response_mask": (torch.arange(R).unsqueeze(0) < rlen.unsqueeze(1)).float(),
                       "old_log_probs": -torch.rand(B, R, generator=g) * 8,
                       "advantages": torch.randn(B, generator=g)}).to(dev)
        sh = ShardedParamActorEngine(tiny_qwen3(), ParallelState(world_size=world, rank=rank, device=dev),
                                     lr=1e-3, seed=3)
        # the resident-weight engine on the same two ranks (plain NCCL collectives)
        ref = ActorEngine(tiny_qwen3(), ParallelState(world_size=world, rank=rank, device=dev), lr=1e-3, seed=3,
                          fused_comm=False)
        n = ref.model.layout.numel
        w_eq = bool(torch.equal(sh.full_flat()[:n], ref.model.flat[:n]))
        lp_s, _ = sh.compute_log_probs(b)
        lp_r, _ = ref.compute_log_probs(b)
        m = b.tensors["response_mask"] > 0
        lp_err = float((lp_s - lp_r)[m].abs().max())
        gs = sh.update_policy(b, GRPOConfig(), "grpo", rows_per_micro=2)["actor/grad_norm"]
        gr = ref.update_policy(b, GRPOConfig(), "grpo", rows_per_micro=2)["actor/grad_norm"]
        w1 = sh.full_flat()[:n].float()
        dw = float((w1 - ref.model.flat[:n].float()).abs().max())
        q.put((rank, {"w_eq": w_eq, "lp_err": lp_err, "gs": gs, "gr": gr, "dw": dw}))
    except Exception as e:
        import traceback
        q.put((rank, {"error": traceback.format_exc()[-2000:] + repr(e)}))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_param_engine_matches_resident_on_gpus():
    """Parameter-sharded engine (NCCL gathers / reduce-scatters) against the
    resident-weight engine on the same 2 GPUs: equal weights, equal scores,
    the same gradient norm and an update within bf16 rounding."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28300 + os.getpid() % 150
    procs = [ctx.Process(target=_sharded_engine_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert "error" not in v, v["error"]
        assert v["w_eq"], r
        assert v["lp_err"] < 2e-2, (r, v)
        assert abs(v["gs"] - v["gr"]) < 2e-2 * v["gr"], (r, v)
        assert v["dw"] < 5e-3, (r, v)        # lr 1e-3: one Adam step moves weights by ~1e-3


def _rollout_tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=_PG_TIMEOUT)
    try:
        from lumenrl_b200.engine.inference.engine import RolloutEngine, SamplingParams
        from lumenrl_b200.models.config import tiny_qwen3
        from lumenrl_b200.models.qwen3 import Qwen3Model
        dev = torch.device("cuda", rank)
        m = Qwen3Model(tiny_qwen3(), device=dev, dtype=torch.bfloat16, requires_grad=False)
        m.init_weights(5)
        sp = SamplingParams(max_new_tokens=24, n=4, seed=3, stop_at_eos=False)
        prompts = [[5 + i for i in range(70)], [11 + i for i in range(33)]]
        tp = RolloutEngine(m, max_num_seqs=8, max_model_len=160, tp_group=dist.group.WORLD)
        assert not tp.use_cuda_graph          # TP decode runs eagerly
        out = tp.generate(prompts, sp)
        one = RolloutEngine(m, max_num_seqs=8, max_model_len=160, use_cuda_graph=True).generate(prompts, sp)
        toks = out.responses.cpu()
        both = [torch.zeros_like(toks) for _ in range(world)]
        dist.all_gather(both, out.responses)
        q.put((rank, {"ranks_agree": all(torch.equal(both[0].cpu(), t.cpu()) for t in both),
                      "same_as_tp1": float((toks == one.responses.cpu()).float().mean()),
                      "lp_gap": float((out.logprobs - one.logprobs).abs()[:, :1].max())}))
    except Exception as e:
        import traceback
        q.put((rank, {"error": traceback.format_exc()[-2000:] + repr(e)}))
    dist.barrier()
    dist.destroy_process_group()


def test_rollout_tp2_on_gpus():
    """TP=2 rollout on 2 GPUs (eager decode step, NCCL all-reduces): both ranks
    draw the same samples, which agree with one GPU's up to bf16
    reduction-order ties."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28450 + os.getpid() % 150
    procs = [ctx.Process(target=_rollout_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert "error" not in v, v["error"]
        assert v["ranks_agree"], r
        assert v["same_as_tp1"] > 0.8, (r, v)
        assert v["lp_gap"] < 5e-2, (r, v)
