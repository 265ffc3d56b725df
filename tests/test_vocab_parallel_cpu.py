"""Vocabulary-parallel token log-probs and entropy on 2 gloo CPU ranks (each
holding half of the LM-head rows, an uneven split) against the full fp32
log-softmax: values, input gradient and each rank's weight-slice gradient."""

import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

T, H, V = 37, 64, 103


def _data():
    g = torch.Generator().manual_seed(0)
    h = torch.randn(T, H, generator=g)
    w = torch.randn(V, H, generator=g) / 8
    tgt = torch.randint(0, V, (T,), generator=g)
    c1, c2 = torch.randn(T, generator=g), torch.randn(T, generator=g)
    return h, w, tgt, c1, c2


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lumenrl_b200.parallel.vocab_parallel import vocab_parallel_token_logprob, vocab_slice
        h, w, tgt, c1, c2 = _data()
        a, b = vocab_slice(V, rank, world)
        hh = h.clone().requires_grad_(True)
        ws = w[a:b].clone().requires_grad_(True)
        logp, ent = vocab_parallel_token_logprob(hh, ws, tgt, a, want_entropy=True, temperature=0.7, rows=16)
        ((logp * c1).sum() + (ent * c2).sum()).backward()
        q.put((rank, {"logp": logp.detach().numpy(), "ent": ent.detach().numpy(), "dh": hh.grad.numpy(),
                      "dw": ws.grad.numpy(), "a": a, "b": b}))
    except Exception as e:
        import traceback
        q.put((rank, {"error": traceback.format_exc()[-2000:] + repr(e)}))
    dist.destroy_process_group()


def test_vocab_parallel_logprob_entropy_and_grads():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29550 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    h, w, tgt, c1, c2 = _data()
    hh, ww = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
    lp_all = torch.log_softmax((hh @ ww.t()) / 0.7, -1)
    logp = lp_all.gather(1, tgt[:, None]).squeeze(1)
    ent = -(lp_all.exp() * lp_all).sum(-1)
    ((logp * c1).sum() + (ent * c2).sum()).backward()
    for r in (0, 1):
        v = res[r]
        assert "error" not in v, v["error"]
        assert abs(torch.from_numpy(v["logp"]) - logp.detach()).max() < 1e-4
        assert abs(torch.from_numpy(v["ent"]) - ent.detach()).max() < 1e-4
        assert abs(torch.from_numpy(v["dh"]) - hh.grad).max() < 1e-4
        assert abs(torch.from_numpy(v["dw"]) - ww.grad[v["a"]: v["b"]]).max() < 1e-4
