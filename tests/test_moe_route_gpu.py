"""Device MoE routing (softmax + top-k + replay + permutation, and its
backward) against the PyTorch router of models/moe.py."""

import pytest
import torch

from lumenrl_b200.models import moe

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,H,E,k,norm", [(257, 64, 8, 2, True), (1000, 128, 128, 8, True), (33, 64, 60, 4, False),
                                          (512, 64, 300, 6, True)])
def test_route_device_matches_torch(cuda, T, H, E, k, norm):
    torch.manual_seed(T + E)
    h = torch.randn(T, H, device=cuda)
    wr = (torch.randn(E, H, device=cuda) / H ** 0.5).requires_grad_(True)
    wr2 = wr.detach().clone().requires_grad_(True)
    ids, w, probs, order, token_of, offs, counts = moe.route_device(h, wr, k, norm)
    rid, rw, rprobs = moe.route(h, wr2, k, norm)
    assert torch.allclose(probs, rprobs, atol=1e-6, rtol=1e-5)
    assert torch.equal(ids.sort(-1).values, rid.sort(-1).values)
    # same weights per (token, expert)
    a = torch.zeros(T, E, device=cuda).scatter(1, ids, w)
    b = torch.zeros(T, E, device=cuda).scatter(1, rid, rw)
    assert torch.allclose(a, b, atol=1e-6, rtol=1e-5)
    # permutation: offsets bound each expert's rows, every pair exactly once
    ref_counts = torch.bincount(rid.reshape(-1), minlength=E)
    assert torch.equal(counts.long(), ref_counts)
    assert torch.equal(offs[1:].long(), torch.cumsum(ref_counts, 0)) and int(offs[0]) == 0
    flat = ids.reshape(-1)
    assert torch.equal(order.sort().values, torch.arange(T * k, device=cuda))
    for e in range(E):
        rows = order[int(offs[e]):int(offs[e + 1])]
        assert bool((flat[rows] == e).all())
    assert torch.equal(token_of, order // k)
    # backward through the weights and the probabilities
    gw, gp = torch.randn(T, k, device=cuda), torch.randn(T, E, device=cuda)
    ((w * gw).sum() + (probs * gp).sum()).backward()
    # torch reference with the same pairing of weight gradients to experts
    gw_e = torch.zeros(T, E, device=cuda).scatter(1, ids, gw)
    gw_r = gw_e.gather(1, rid)
    ((rw * gw_r).sum() + (rprobs * gp).sum()).backward()
    assert torch.allclose(wr.grad, wr2.grad, atol=1e-4, rtol=1e-3)


def test_route_device_replay(cuda):
    torch.manual_seed(0)
    T, H, E, k = 64, 32, 16, 2
    h = torch.randn(T, H, device=cuda)
    wr = torch.randn(E, H, device=cuda) / H ** 0.5
    replay = torch.randint(0, E, (T, k), device=cuda)
    replay[::3] = -1                       # rows without a rollout decision keep the live choice
    ids, w, probs, *_ = moe.route_device(h, wr, k, True, replay)
    rid, rw, _ = moe.route(h, wr, k, True, replay)
    assert torch.equal(ids, torch.where((replay >= 0).all(-1, keepdim=True), replay, ids))
    a = torch.zeros(T, E, device=cuda).scatter_add(1, ids, w)
    b = torch.zeros(T, E, device=cuda).scatter_add(1, rid, rw)
    assert torch.allclose(a, b, atol=1e-6)
