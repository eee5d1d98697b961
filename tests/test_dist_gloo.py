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


def _gpt_small_shapes():
    muon = [torch.empty(s) for _ in range(8) for s in [(512, 512)] * 4 + [(2048, 512), (512, 2048), (64, 64)]]
    adam = [(1, torch.empty(50304, 512)), (2, torch.empty(50304, 512))] + \
           [(2, torch.empty(512)) for _ in range(17)] + [(2, torch.empty(64)) for _ in range(8)]
    return muon, adam


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_layout_partitions_every_element_once(world):
    """Every AdamW element and every Muon matrix belongs to exactly one rank; the packed chunks do not
    overlap; AdamW slices are equal and the Newton-Schulz load is balanced (the gpt-small shapes)."""
    from rgpt_b200.optimizer import ShardLayout

    muon, adam = _gpt_small_shapes()
    lay = ShardLayout(muon, adam, world)
    seen = {}
    covered = torch.zeros(world * lay.C, dtype=torch.int32)
    for r in range(world):
        for t, _, off, lo, n in lay.segments([r], lambda p: p):
            assert r * lay.C <= off and off + n <= (r + 1) * lay.C
            covered[off:off + n] += 1
            seen.setdefault(id(t), []).append((lo, lo + n))
    assert int(covered.max()) == 1
    for p in muon + [p for _, p in adam]:
        ranges = sorted(seen[id(p)])
        assert ranges[0][0] == 0 and ranges[-1][1] == p.numel()
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))  # contiguous, no gaps or overlaps
    assert sum(len(lay.owned_muon(r)) for r in range(world)) == len(muon)
    cost = lambda p: 2 * min(p.shape) ** 2 * max(p.shape) * 2 + 2 * min(p.shape) ** 3  # noqa: E731
    load = [sum(cost(p) for p in lay.owned_muon(r)) for r in range(world)]
    assert max(load) <= 1.01 * min(load)
    assert lay.S * world >= lay.adam_total and lay.S % 8 == 0 and lay.C % 8 == 0


def _protocol_worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from rgpt_b200.optimizer import ShardLayout

        g0 = torch.Generator().manual_seed(0)
        muon = [torch.randn(*s, generator=g0) for s in [(64, 32), (32, 32), (16, 48), (40, 8)]]
        adam = [(1, torch.randn(37, generator=g0)), (2, torch.randn(5, generator=g0)), (2, torch.randn(10, 3, generator=g0))]
        params = muon + [p for _, p in adam]
        grads = {id(p): torch.randn(p.shape, generator=torch.Generator().manual_seed(100 * rank + i))
                 for i, p in enumerate(params)}
        lay = ShardLayout(muon, adam, world)

        def pack(segs, buf, of):
            for t, _, off, lo, n in segs:
                buf[off:off + n] = of(t).reshape(-1)[lo:lo + n]

        def unpack(segs, buf, of):
            for t, _, off, lo, n in segs:
                of(t).reshape(-1)[lo:lo + n] = buf[off:off + n]

        # 1. reduce-scatter of the packed gradients; each rank unpacks its own chunk
        send = torch.zeros(world * lay.C)
        pack(lay.segments(range(world), lambda p: p), send, lambda t: grads[id(t)])
        recv = torch.zeros(lay.C)
        dist.reduce_scatter_tensor(recv, send, op=dist.ReduceOp.SUM)
        recv /= world
        avg = {k: torch.zeros_like(v) for k, v in grads.items()}
        unpack(lay.segments([rank], lambda p: p, base_of=lambda r: 0), recv, lambda t: avg[id(t)])
        # the true average on the owned parts
        full = {k: v.clone() for k, v in grads.items()}
        for v in full.values():
            dist.all_reduce(v)
            v /= world
        ok_rs = all(torch.allclose(avg[id(t)].reshape(-1)[lo:lo + n], full[id(t)].reshape(-1)[lo:lo + n])
                    for t, _, _, lo, n in lay.segments([rank], lambda p: p, base_of=lambda r: 0))
        # 2. "update" the owned parts (p -= avg grad), 3. all-gather and unpack everywhere
        for t, _, _, lo, n in lay.segments([rank], lambda p: p, base_of=lambda r: 0):
            t.reshape(-1)[lo:lo + n] -= avg[id(t)].reshape(-1)[lo:lo + n]
        s32 = torch.zeros(lay.C)
        pack(lay.segments([rank], lambda p: p, base_of=lambda r: 0), s32, lambda t: t)
        r32 = torch.zeros(world * lay.C)
        dist.all_gather_into_tensor(r32, s32)
        unpack(lay.segments(range(world), lambda p: p), r32, lambda t: t)
        g1 = torch.Generator().manual_seed(0)
        init = [torch.randn(*s, generator=g1) for s in [(64, 32), (32, 32), (16, 48), (40, 8)]] + \
               [torch.randn(37, generator=g1), torch.randn(5, generator=g1), torch.randn(10, 3, generator=g1)]
        ok_ag = all(torch.allclose(p, i - full[id(p)], atol=1e-6) for p, i in zip(params, init))
        q.put((rank, bool(ok_rs), bool(ok_ag)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_step_protocol_over_gloo_ranks(world):
    """The sharded data-parallel step's data movement on CPU ranks: packed owner-major gradients through a
    reduce-scatter give each rank the average of what it owns; the owners' updates through an all-gather
    give every rank the same, fully updated parameters."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_protocol_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok_rs and ok_ag for _, ok_rs, ok_ag in res), res
