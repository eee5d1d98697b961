"""Muon / AdamW kernels over several steps vs the CPU oracle (optimizer.py of the reference).

Multi-step checks matter: momentum_buffer is bf16 state carried across steps,
and Newton-Schulz is scale-invariant, so a lost momentum would be invisible in
one step. Tolerances: momentum buffers within 1e-2 (bf16 lerp rounding), AdamW
weights within 1e-5, Muon weight deltas within 5e-2 (bf16 Newton-Schulz), bf16
shadows equal to bf16(weights).
"""
import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200.optimizer import Muon, muon_update, zeropower_via_newtonschulz5

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("shape", [(256, 128), (128, 384), (64, 64), (2, 512)])
def test_muon_multi_step_momentum_and_weights(cuda, shape):
    g = torch.Generator().manual_seed(sum(shape))
    w0 = torch.randn(*shape, generator=g) * 0.02
    b0 = torch.randn(shape[0], generator=g) * 0.1 + 1.0
    grads = [(torch.randn(*shape, generator=g) * 1e-2, torch.randn(shape[0], generator=g) * 1e-3) for _ in range(3)]
    W = torch.nn.Parameter(w0.clone().to(cuda))
    Bv = torch.nn.Parameter(b0.clone().to(cuda))
    W._rgpt_shadow = torch.zeros(shape, device=cuda, dtype=torch.bfloat16)
    opt = Muon([{"params": [W], "use_muon": True}, {"params": [Bv], "use_muon": False, "weight_decay": 0.0}],
               lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    ow = {"w": w0.clone(), "b": b0.clone()}
    oopt = O.OracleMuon(ow, lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    oopt.groups = (["w"], [], ["b"])
    for gw, gb in grads:
        W.grad = gw.to(cuda)
        Bv.grad = gb.to(cuda)
        opt.step()
        oopt.step({"w": gw, "b": gb})
    torch.cuda.synchronize()
    m_ours = opt.state[W]["momentum_buffer"].float().cpu()
    m_ref = oopt.state["w"]["momentum_buffer"].float()
    assert rel(m_ours, m_ref) < 1e-2
    assert rel(W.detach().cpu() - w0, ow["w"] - w0) < 5e-2
    assert rel(Bv.detach().cpu() - b0, ow["b"] - b0) < 1e-5
    assert torch.equal(W._rgpt_shadow, W.detach().to(torch.bfloat16))
    assert opt.param_groups[1]["_adam_step"] == 3


def test_zeropower_bf16_vs_reference_rounding_and_fp32(cuda):
    g = torch.Generator().manual_seed(5)
    for shape in [(512, 2048), (2048, 512), (512, 512), (64, 64)]:
        G = torch.randn(*shape, generator=g) * 1e-2
        ours = zeropower_via_newtonschulz5(G.to(cuda), 5).float().cpu()
        ref16 = O.zeropower_ns5(G, 5, dtype=torch.bfloat16).float()
        ref32 = O.zeropower_ns5(G, 5, dtype=torch.float32)
        # bf16 iteration: same math, rounding fused differently from the reference's op-by-op bf16
        assert rel(ours, ref16) < 5e-2, shape
        assert rel(ours, ref32) < 5e-2, shape


def test_muon_update_functional_matches_oracle(cuda):
    g = torch.Generator().manual_seed(9)
    G1, G2 = torch.randn(96, 32, generator=g) * 1e-2, torch.randn(96, 32, generator=g) * 1e-2
    m = torch.zeros(96, 32, dtype=torch.bfloat16, device=cuda)
    mr = torch.zeros(96, 32, dtype=torch.bfloat16)
    for G in (G1, G2):
        u = muon_update(G.to(cuda), m, 0.95, 5, True, O.muon_scale(96, 32))
        ur = O.muon_update(G, mr, 0.95, 5, True, O.muon_scale(96, 32))
        assert rel(u.float(), ur.float()) < 5e-2
        assert rel(m.float(), mr.float()) < 1e-2
