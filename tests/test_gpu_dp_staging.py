"""The sharded data-parallel step's single-GPU pieces: the staging kernel and AdamW over element slices.

rgpt_segment_copy packs a ShardLayout's segments (every rank's chunk, as the gradient reduce-scatter
needs them) and unpacks them again, with fp32 and bf16 buffers and the bf16 GEMM copies; AdamW run over
the slices two ranks own equals AdamW over the whole tensors. Both must be exact: they are copies and
the same elementwise arithmetic.
"""
import pytest
import torch

from rgpt_b200 import native as nv
from rgpt_b200.optimizer import Muon, ShardLayout

pytestmark = pytest.mark.gpu


def _params(dev):
    g = torch.Generator().manual_seed(0)
    muon = [torch.nn.Parameter(torch.randn(*s, generator=g).to(dev)) for s in [(512, 512), (2048, 512), (64, 64)]]
    adam = [(1, torch.nn.Parameter(torch.randn(512, generator=g).to(dev))),
            (2, torch.nn.Parameter(torch.randn(1000, 64, generator=g).to(dev))),
            (2, torch.nn.Parameter(torch.randn(37, generator=g).to(dev)))]
    return muon, adam


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("buf_dtype", [torch.float32, torch.bfloat16])
def test_segment_copy_pack_unpack(cuda, world, buf_dtype):
    muon, adam = _params(cuda)
    lay = ShardLayout(muon, adam, world)
    params = muon + [p for _, p in adam]
    buf = torch.full((world * lay.C,), -7.0, device=cuda, dtype=buf_dtype)
    nv.segment_copy(nv.segment_table(lay.segments(range(world), lambda p: p), cuda), buf, tensor_bf16=False,
                    scale=0.5)
    # the reference packing, by slicing
    ref = torch.full_like(buf, -7.0)
    for t, _, off, lo, n in lay.segments(range(world), lambda p: p):
        ref[off:off + n] = (0.5 * t.detach().reshape(-1)[lo:lo + n]).to(buf_dtype)
    assert torch.equal(buf, ref)
    # unpack every chunk into fresh tensors and bf16 copies
    outs = {id(p): torch.zeros_like(p) for p in params}
    copies = {id(p): torch.zeros(p.shape, device=cuda, dtype=torch.bfloat16) for p in params}
    plan = nv.segment_table(lay.segments(range(world), lambda p: outs[id(p)], second_of=lambda p: copies[id(p)]), cuda)
    nv.segment_copy(plan, buf, tensor_bf16=False, scale=2.0, unpack=True)
    for p in params:
        want = (0.5 * p.detach()).to(buf_dtype).float() * 2.0
        assert torch.equal(outs[id(p)], want), tuple(p.shape)
        assert torch.equal(copies[id(p)], want.bfloat16()), tuple(p.shape)
    # one rank's own chunk, at offset 0 of a chunk-sized buffer
    r = world - 1
    own = torch.zeros(lay.C, device=cuda, dtype=buf_dtype)
    nv.segment_copy(nv.segment_table(lay.segments([r], lambda p: p, base_of=lambda _: 0), cuda), own,
                    tensor_bf16=False)
    for t, _, off, lo, n in lay.segments([r], lambda p: p, base_of=lambda _: 0):
        assert torch.equal(own[off:off + n], t.detach().reshape(-1)[lo:lo + n].to(buf_dtype))


def test_adamw_over_owned_slices_equals_whole_tensors(cuda):
    _, adam = _params(cuda)
    world = 2
    lay = ShardLayout([], adam, world)
    g = torch.Generator().manual_seed(1)
    grads = [torch.randn(p.shape, generator=g).to(cuda) * 1e-2 for _, p in adam]

    def build():
        ps = [torch.nn.Parameter(p.detach().clone()) for _, p in adam]
        for p, gr in zip(ps, grads):
            p.grad = gr.clone()
        opt = Muon([{"params": ps[:1], "use_muon": False, "weight_decay": 0.0},
                    {"params": ps[1:], "use_muon": False, "weight_decay": 0.1}], lr=1e-3)
        return ps, opt

    whole, opt_w = build()
    sliced, opt_s = build()
    lay_s = ShardLayout([], [(gi, p) for (gi, _), p in zip(adam, sliced)], world)
    for _ in range(3):
        opt_w.step()
        for gi, group in enumerate(opt_s.param_groups):
            slices = [(p, lo, hi) for r in range(world) for g_, p, lo, hi, _ in lay_s.adam_slices(r) if g_ == gi + 1]
            for job in opt_s._adamw_jobs(gi, group, None, slices=slices):
                job()
    torch.cuda.synchronize()
    for a, b in zip(whole, sliced):
        assert torch.equal(a, b), tuple(a.shape)
