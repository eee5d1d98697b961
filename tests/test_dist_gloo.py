"""Data-parallel gradient averaging of DistMuon on two CPU ranks (gloo).

The GPU update itself is covered by the -m gpu tests; this checks the cross-rank step that
DistMuon adds in front of it (the all-reduce of each rank's flat gradient arena and of loose
gradients, divided by the world size), the way the reference's DDP averages gradients
(trainer.py:47-53) before every rank runs the same optimizer update.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from rgpt_b200.optimizer import DistMuon

        # two parameters whose grads are views of one flat arena, and one loose parameter
        arena = torch.arange(12, dtype=torch.float32) * (rank + 1)
        p1 = torch.nn.Parameter(torch.zeros(2, 3))
        p2 = torch.nn.Parameter(torch.zeros(6))
        p1.grad = arena[:6].view(2, 3)
        p2.grad = arena[6:]
        p1._rgpt_grad_arena = arena
        p2._rgpt_grad_arena = arena
        p3 = torch.nn.Parameter(torch.zeros(4))
        p3.grad = torch.full((4,), float(rank + 1))
        opt = DistMuon([dict(params=[p1, p2], use_muon=True), dict(params=[p3], use_muon=False)])
        opt._average_grads()
        mean = (1 + world) / 2.0  # ranks scale by rank + 1
        ok = (torch.allclose(arena, torch.arange(12, dtype=torch.float32) * mean) and
              torch.allclose(p3.grad, torch.full((4,), mean)) and
              p1.grad.data_ptr() == arena.data_ptr())  # the views still alias the arena
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_distmuon_averages_grads_over_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def test_ns_owner_assignment_is_balanced_and_deterministic():
    from rgpt_b200.optimizer import assign_ns_owners

    # gpt-small Muon matrices as NS sees them: 4 x [512,512] and 2 x [512,2048] per layer, gate [64,64]
    shapes = ([(512, 512)] * 4 + [(512, 2048)] * 2 + [(64, 64)]) * 8
    cost = [2 * r * r * c * 2 + 2 * r ** 3 for r, c in shapes]
    for world in (1, 2, 4, 8):
        own = assign_ns_owners(shapes, world)
        assert own == assign_ns_owners(shapes, world)
        assert set(own) == set(range(world))
        load = [sum(c for c, o in zip(cost, own) if o == r) for r in range(world)]
        assert max(load) <= 1.01 * min(load)
