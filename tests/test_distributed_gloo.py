"""Data-parallel host logic on CPU: two gloo ranks (127.0.0.1).

Checks the pieces the multi-GPU bench and training rely on:

* the Trainer's DDP wrapping (eager, per-parameter layout) averages
  gradients so both ranks hold identical parameters after a step, equal to a
  single-process step on the averaged gradient;
* the flat-buffer path the captured multi-GPU step uses (parameters as views
  of one flat buffer, rank 0's parameters broadcast at construction, one
  all-reduce of the flat gradients, or bucketed all-reduces launched from
  gradient hooks during the backward) gives the same parameters, on ranks
  that were initialised differently;
* max_over_ranks reports the slowest rank's time.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


class _Toy(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(8, 4)

    def forward(self, mix, target):
        return (self.lin(mix) - target).abs().mean()


class _Deep(torch.nn.Module):
    """Three layers used in order, so their gradients become final in reverse order during the backward."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(8, 16)
        self.b = torch.nn.Linear(16, 16)
        self.c = torch.nn.Linear(16, 4)

    def forward(self, mix, target):
        return (self.c(torch.tanh(self.b(torch.tanh(self.a(mix))))) - target).abs().mean()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pymsst_b200.train import Trainer, max_over_ranks

        torch.manual_seed(0)
        trainer = Trainer(_Toy(), lr=1e-2, distributed=True, device=torch.device("cpu"))
        g = torch.Generator().manual_seed(100 + rank)
        mix, tgt = torch.randn(16, 8, generator=g), torch.randn(16, 4, generator=g)
        trainer.step(mix, tgt)
        params = torch.cat([p.detach().flatten() for p in trainer.model.parameters()])
        gathered = [torch.empty_like(params) for _ in range(world)]
        dist.all_gather(gathered, params)
        worst = max_over_ranks([float(rank + 1), 10.0 * (world - rank)], torch.device("cpu"))
        out[rank] = (params.tolist(), [t.tolist() for t in gathered], worst)
    finally:
        dist.destroy_process_group()


def test_ddp_two_gloo_ranks_average_gradients():
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    p0, gathered, worst = out[0]
    assert gathered[0] == gathered[1], "ranks hold different parameters after a DDP step"
    assert worst == [2.0, 20.0]
    # single-process reference: the same step on the mean of the two ranks' gradients
    torch.manual_seed(0)
    model = _Toy()
    opt = torch.optim.Adam(model.parameters(), lr=1e-2)
    grads = []
    for rank in range(world):
        model.zero_grad()
        g = torch.Generator().manual_seed(100 + rank)
        mix, tgt = torch.randn(16, 8, generator=g), torch.randn(16, 4, generator=g)
        model(mix, tgt).backward()
        grads.append([p.grad.clone() for p in model.parameters()])
    for p, *gs in zip(model.parameters(), *grads):
        p.grad = sum(gs) / world
    opt.step()
    ref = torch.cat([p.detach().flatten() for p in model.parameters()])
    torch.testing.assert_close(torch.tensor(p0), ref, rtol=1e-6, atol=1e-6)


def _flat_worker(rank, world, port, out, overlap):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pymsst_b200.train import Trainer

        torch.manual_seed(7 + rank)  # different initial weights on each rank: the trainer must broadcast rank 0's
        model = _Deep()
        # a bucket per parameter (tiny cap) so the overlapped path launches several all-reduces mid-backward
        trainer = Trainer(model, lr=1e-2, distributed=True, device=torch.device("cpu"), flat_params=True,
                          overlap_allreduce=overlap, bucket_cap_mb=1e-4)
        assert trainer.flat and trainer.flat_param is not None
        for step in range(3):
            g = torch.Generator().manual_seed(100 * step + rank)
            mix, tgt = torch.randn(16, 8, generator=g), torch.randn(16, 4, generator=g)
            trainer.step(mix, tgt)
        params = torch.cat([p.detach().flatten() for p in model.parameters()])
        gathered = [torch.empty_like(params) for _ in range(world)]
        dist.all_gather(gathered, params)
        out[rank] = ([t.tolist() for t in gathered], len(trainer._buckets), trainer.bucket_launches)
        trainer.close()  # hooks removed: a further backward launches no all-reduce
        model(torch.randn(2, 8), torch.randn(2, 4)).backward()
        assert trainer.bucket_launches == out[rank][2]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("overlap", [False, True])
def test_flat_gradient_allreduce_two_gloo_ranks(overlap):
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_flat_worker, args=(world, _free_port(), out, overlap), nprocs=world, start_method="spawn",
                       join=True)
    gathered, buckets, launches = out[0]
    assert gathered[0] == gathered[1], "ranks hold different parameters after flat all-reduce steps"
    if overlap:
        # six parameters, one bucket each, each all-reduced from its gradient hook in each of the three steps
        assert buckets == 6 and launches == 18
    else:
        assert launches == 0
    # single-process reference: rank 0's initial weights, three Adam steps on the mean of both ranks' gradients
    torch.manual_seed(7)
    model = _Deep()
    opt = torch.optim.Adam(model.parameters(), lr=1e-2)
    for step in range(3):
        grads = []
        for rank in range(world):
            model.zero_grad()
            g = torch.Generator().manual_seed(100 * step + rank)
            mix, tgt = torch.randn(16, 8, generator=g), torch.randn(16, 4, generator=g)
            model(mix, tgt).backward()
            grads.append([p.grad.clone() for p in model.parameters()])
        for p, *gs in zip(model.parameters(), *grads):
            p.grad = sum(gs) / world
        opt.step()
    ref = torch.cat([p.detach().flatten() for p in model.parameters()])
    torch.testing.assert_close(torch.tensor(gathered[0]), ref, rtol=1e-5, atol=1e-6)
