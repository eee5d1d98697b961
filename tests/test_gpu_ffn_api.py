"""FusedLinearActivationFunction.apply (the public op, model/kernels.py:289-374) on CUDA.

1. Against the reference's own Triton kernels: tests/golden/ffn.pt holds their outputs (run under
   the Triton interpreter by tests/golden/gen_golden.py) for X [64, 64], W1 [128, 64], W2 [128, 32]
   and the loss y.sum(), for all four activations.
2. At the fused linear+activation sweep's shapes (X [M, 512] ~ N(0, 1), W1 and W2 [2048, 512]
   ~ N(0, 0.02), upstream gradient ~ N(0, 1)) against a plain PyTorch fp32 composite
   act(X W1^T) W2 of the same bf16-rounded inputs and its autograd gradients.

Tolerance: the op computes with bf16 operands, bf16 pre/post activations and fp32 accumulation,
so outputs and gradients carry a few bf16 roundings: 1e-2 relative Frobenius error for the output
and 2e-2 for the gradients against the reference Triton outputs (which ran in fp32), 1e-2 for every
tensor against the fp32 composite of the bf16-rounded inputs.
"""
import os

import pytest
import torch

from rgpt_b200.model import FeedForward, FusedLinearActivationFunction
from rgpt_b200.model.config import Config
from rgpt_b200.workloads import FFN_SWEEP

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ACTS = ["squared_relu", "gelu", "silu", "mish"]


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def torch_act(name, x):
    import torch.nn.functional as F
    if name == "squared_relu":
        return torch.relu(x) ** 2
    if name == "gelu":
        return F.gelu(x, approximate="tanh")
    if name == "silu":
        return F.silu(x)
    return F.mish(x)


@pytest.mark.parametrize("act", ACTS)
def test_apply_matches_reference_triton_golden(cuda, act):
    g = torch.load(os.path.join(GOLD, "ffn.pt"), weights_only=False)
    x, w1, w2 = (g[k].to(cuda).requires_grad_(True) for k in ("x", "w1", "w2"))
    y = FusedLinearActivationFunction.apply(x, w1, w2, act)
    assert y.dtype == torch.float32 and y.shape == g[act]["y"].shape
    y.sum().backward()
    r = g[act]
    assert rel(y, r["y"]) < 1e-2, rel(y, r["y"])
    assert rel(x.grad, r["dx"]) < 2e-2, rel(x.grad, r["dx"])
    assert rel(w1.grad, r["dw1"]) < 2e-2, rel(w1.grad, r["dw1"])
    assert rel(w2.grad, r["dw2"]) < 2e-2, rel(w2.grad, r["dw2"])


def _sweep_case(cuda, M, act, seed):
    K, N = FFN_SWEEP["K"], FFN_SWEEP["N"]
    gen = torch.Generator(device=cuda).manual_seed(seed)
    x = (torch.randn(M, K, device=cuda, generator=gen) * FFN_SWEEP["x_std"]).bfloat16()
    w1 = (torch.randn(N, K, device=cuda, generator=gen) * FFN_SWEEP["w_std"]).bfloat16()
    w2 = (torch.randn(N, K, device=cuda, generator=gen) * FFN_SWEEP["w_std"]).bfloat16()
    dy = torch.randn(M, K, device=cuda, generator=gen).bfloat16()
    xs, a, b = (t.clone().requires_grad_(True) for t in (x, w1, w2))
    y = FusedLinearActivationFunction.apply(xs, a, b, act)
    y.backward(dy)
    xr, ar, br = (t.float().requires_grad_(True) for t in (x, w1, w2))
    yr = torch_act(act, xr @ ar.t()) @ br
    yr.backward(dy.float())
    return (y, xs.grad, a.grad, b.grad), (yr, xr.grad, ar.grad, br.grad)


@pytest.mark.parametrize("act", ACTS)
def test_apply_at_sweep_shape_matches_fp32_composite(cuda, act):
    ours, ref = _sweep_case(cuda, FFN_SWEEP["M"][0], act, seed=5)
    for name, o, r in zip(("y", "dx", "dw1", "dw2"), ours, ref):
        assert o.dtype == torch.bfloat16 and o.shape == r.shape, name
        assert rel(o.float(), r) < 1e-2, (name, rel(o.float(), r))


def test_apply_at_largest_sweep_shape(cuda):
    ours, ref = _sweep_case(cuda, FFN_SWEEP["M"][-1], "squared_relu", seed=6)
    for name, o, r in zip(("y", "dx", "dw1", "dw2"), ours, ref):
        assert rel(o.float(), r) < 1e-2, (name, rel(o.float(), r))


def test_feed_forward_module_forward(cuda):
    """FeedForward.forward (model/feed_forward.py:25-37) on a [B, T, d] input, fp32 parameters."""
    torch.manual_seed(3)
    ff = FeedForward(Config(d_model=512, activation_type="gelu")).to(cuda)
    x = torch.randn(2, 256, 512, device=cuda, requires_grad=True)
    y = ff(x)
    y.square().sum().backward()
    xr = x.detach().clone().requires_grad_(True)
    w1 = ff.fc1.weight.detach().clone().requires_grad_(True)
    w2 = ff.fc2.weight.detach().clone().requires_grad_(True)
    yr = torch_act("gelu", xr @ w1.t()) @ w2.t()
    yr.square().sum().backward()
    assert y.shape == (2, 256, 512)
    assert rel(y, yr) < 1e-2
    assert rel(x.grad, xr.grad) < 2e-2
    assert rel(ff.fc1.weight.grad, w1.grad) < 2e-2
    assert rel(ff.fc2.weight.grad, w2.grad) < 2e-2
