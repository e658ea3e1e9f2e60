"""The multi-rank path on CPU with the gloo backend (world size 2): batch sharding,
max-over-ranks timing, and the data-parallel identity the training path relies
on (per-rank LTHC weight gradients summed over ranks equal the full-batch
gradient).  The weight-gradient arithmetic is the oracle's."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from flowmatching_lthc_b200 import dist as D


def test_shard_bounds_cover_exactly():
    for total in (0, 1, 7, 64, 1024):
        for world in (1, 2, 3, 8):
            spans = [D.shard(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        D.shard(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from oracle import lthc_oracle as O

    O.set_num_threads(1)
    D.init("gloo", D.Rank(rank, world, rank), timeout_s=60)
    try:
        B, G, C, L = 5, 2, 16, 3
        gen = torch.Generator().manual_seed(123)
        gx = torch.randn(B, 4 * G, 4 * G, C, generator=gen)
        dz = [torch.randn(B, G * G, C, generator=gen) for _ in range(L)]
        a, b = D.shard(B, rank, world)
        local = O.weight_grad(gx[a:b], [d[a:b] for d in dz]).double()
        D.reduce_sum_(local)
        slowest = D.reduce_max(float(rank + 1))
        if rank == 0:
            full = O.weight_grad(gx, dz).double()
            q.put(((local - full).abs().max().item(), full.abs().max().item(), slowest))
        D.barrier()
    finally:
        D.shutdown()


def test_gloo_two_ranks_weight_grad_allreduce_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, scale, slowest = q.get(timeout=5)
    assert err <= 1e-6 * scale
    assert slowest == 2.0


def _flat_worker(rank: int, world: int, port: int, q) -> None:
    """A small model's data-parallel step with FlatGradients: after the one
    all-reduce every rank holds the full-batch mean gradient, which equals what a
    single process computes on the whole batch (the loss is a mean over images)."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    D.init("gloo", D.Rank(rank, world, rank), timeout_s=60)
    try:
        torch.manual_seed(0)
        net = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.SiLU(), torch.nn.Linear(16, 4))
        x = torch.randn(6, 8, generator=torch.Generator().manual_seed(1))
        y = torch.randn(6, 4, generator=torch.Generator().manual_seed(2))
        fg = D.FlatGradients(net.parameters())
        a, b = D.shard(6, rank, world)
        fg.zero_grad()
        ((net(x[a:b]) - y[a:b]).square().mean(1).sum() / (b - a)).backward()
        fg.allreduce()
        got = torch.cat([q.grad.reshape(-1) for q in net.parameters()])
        assert got.data_ptr() != 0 and all(q.grad.data_ptr() >= fg.flat.data_ptr() for q in net.parameters())
        ref = [torch.zeros_like(q) for q in net.parameters()]
        for i in range(6):  # the full batch on one process: mean over images of the per-image loss
            g = torch.autograd.grad((net(x[i:i + 1]) - y[i:i + 1]).square().mean(), list(net.parameters()))
            ref = [r + gi / 6 for r, gi in zip(ref, g)]
        want = torch.cat([r.reshape(-1) for r in ref])
        if rank == 0:
            q.put((got - want).abs().max().item())
        D.barrier()
    finally:
        D.shutdown()


def test_gloo_flat_gradient_allreduce_equals_the_full_batch_gradient():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_flat_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) < 1e-6
