"""tcgen05 causal attention (rgpt_attn_*) against a plain PyTorch fp32 reference.

Inputs are bf16 (q, k, v, gate, upstream grad); the reference runs the same
bf16 values in fp32. Tolerances (rel. Frobenius): forward outputs 1e-2, lse
1e-4 (absolute, natural log), gradients 2e-2 (P and dS are rounded to bf16
before their MMAs, as in any bf16 flash attention).
"""
import math

import pytest
import torch

from rgpt_b200 import native as nv

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def make_inputs(B, T, H, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    d = H * 64
    qkv = torch.randn(B * T, 3 * d, device=dev, generator=g).bfloat16()
    qk = torch.randn(B * T, 2 * d, device=dev, generator=g).bfloat16()
    gate = torch.sigmoid(torch.randn(B * T, d, device=dev, generator=g)).bfloat16()
    return qk, qkv, gate


def reference(qk, qkv, gate, B, T, H):
    d = H * 64
    q = qk[:, :d].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    k = qk[:, d:].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    v = qkv[:, 2 * d:].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(64)
    s = s.masked_fill(torch.ones(T, T, device=q.device, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ v
    o_tok = o.transpose(1, 2).reshape(B * T, d)
    return q, k, v, o_tok, lse


@pytest.mark.parametrize("B,T,H", [(2, 256, 2), (1, 1023, 4), (2, 200, 1), (3, 77, 2), (16, 1024, 8)])
def test_attention_fwd_bwd(cuda, B, T, H):
    d = H * 64
    qk, qkv, gate = make_inputs(B, T, H, cuda, 7 + T)
    o = torch.empty(B * T, d, device=cuda, dtype=torch.bfloat16)
    og = torch.empty_like(o)
    lse = torch.empty(B, H, T, device=cuda, dtype=torch.float32)
    nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H)
    q, k, v, o_ref, lse_ref = reference(qk, qkv, gate, B, T, H)
    assert rel_err(o, o_ref) < 1e-2
    assert rel_err(og, o_ref * gate.float()) < 1e-2
    assert (lse - lse_ref).abs().max().item() < 1e-3

    # backward through og = o * gate
    g = torch.Generator(device=cuda).manual_seed(99)
    dog = torch.randn(B * T, d, device=cuda, generator=g).bfloat16()
    do = torch.empty_like(o)
    dgp = torch.empty_like(o)
    D = torch.empty(B, H, T, device=cuda, dtype=torch.float32)
    dq = torch.full((B * T, d), 7.0, device=cuda, dtype=torch.float32)  # zeroed by the prep pass
    nv.attn_bwd_prep(dog, o, gate, do, dgp, D, B, T, H, dq_zero=dq)
    dk = torch.empty(B * T, d, device=cuda, dtype=torch.float32)
    dqkv = torch.zeros(B * T, 3 * d, device=cuda, dtype=torch.bfloat16)
    nv.attn_bwd(qk, qkv, do, lse, D, dq, dk, dqkv[:, 2 * d:], B, T, H)
    torch.cuda.synchronize()

    gf = gate.float()
    (o_ref * gf * dog.float()).sum().backward()
    tok = lambda t: t.transpose(1, 2).reshape(B * T, d)
    assert rel_err(dq, tok(q.grad)) < 2e-2
    assert rel_err(dk, tok(k.grad)) < 2e-2
    assert rel_err(dqkv[:, 2 * d:], tok(v.grad)) < 2e-2
    # gate path: d(pre-sigmoid) = dog * o * g * (1 - g)
    assert rel_err(dgp, dog.float() * o_ref.detach() * gf * (1 - gf)) < 2e-2
    assert rel_err(do, dog.float() * gf) < 1e-2
    assert dqkv[:, :2 * d].abs().max().item() == 0.0  # untouched columns stay zero


def test_attention_rejects_bad_head_dim(cuda):
    qk = torch.zeros(8, 2 * 96, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        nv.attn_fwd(qk, qk, None, qk, None, torch.zeros(8, device=cuda), 1, 8, 1)
