"""DistMuon on two GPUs (NCCL): sharded Newton-Schulz equals the replicated update.

Each rank holds different gradients for the gpt-small Muon shapes ([512,512], [2048,512],
[512,2048], [64,64]) plus an AdamW vector. DistMuon averages them (fp32 all-reduce, as the
reference's DDP does, trainer.py:47-53), then either runs every matrix's Newton-Schulz on every
rank (shard_ns=False, the reference's DistMuon, optimizer.py:317-415) or on one owner rank with
an all-gather of the bf16 results (shard_ns=True). Both must give the same parameters on every
rank (tolerance 1e-6 relative: the NS GEMMs accumulate each matrix in the same order either way).
Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from rgpt_b200.optimizer import DistMuon

        shapes = [(512, 512)] * 4 + [(2048, 512), (512, 2048), (64, 64)]
        g0 = torch.Generator().manual_seed(0)
        init = [torch.randn(*s, generator=g0) * 0.02 for s in shapes] + [torch.ones(512)]
        gr = torch.Generator().manual_seed(100 + rank)
        grads = [torch.randn(t.shape, generator=gr) * 1e-2 for t in init]

        def make(shard):
            ps = [torch.nn.Parameter(t.clone().to(dev)) for t in init]
            for p, g in zip(ps, grads):
                p.grad = g.clone().to(dev)
            groups = [dict(params=ps[:-1], use_muon=True, lr=0.02, weight_decay=0.01),
                      dict(params=ps[-1:], use_muon=False, lr=0.001, weight_decay=0.0)]
            return ps, DistMuon(groups, shard_ns=shard, muon_lr_multiplier=1.0)

        pa, oa = make(True)
        pb, ob = make(False)
        for _ in range(2):  # two steps: momentum carries over
            oa.step()
            ob.step()
            for p, g in zip(pa, grads):
                p.grad.copy_(g.to(dev))
            for p, g in zip(pb, grads):
                p.grad.copy_(g.to(dev))
        torch.cuda.synchronize()
        errs = [((a - b).norm() / b.norm()).item() for a, b in zip(pa, pb)]
        # every rank ends with the same parameters
        ref = [p.detach().clone() for p in pa]
        for t in ref:
            dist.broadcast(t, 0)
        same = max(((a - r).abs().max().item() for a, r in zip(pa, ref)), default=0.0)
        moved = ((pa[0] - init[0].to(dev)).norm() / init[0].norm()).item()
        q.put((rank, max(errs), same, moved))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_distmuon_sharded_ns_matches_replicated_on_two_gpus():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err, same, moved in res:
        assert err < 1e-6, (rank, err)
        assert same == 0.0, (rank, same)
        assert moved > 1e-3, (rank, moved)  # the update did something
