"""The reference's submodules called on their own (model/__init__.py exports), on the native kernels.

RotaryEmbedding.forward (model/rope.py:38-57), the norm modules and functional norms
(model/norm.py:8-162), QKNorm.forward (:200-204), Attention.forward (model/attention.py:35-64) and
TransformerBlock.forward (model/transformer_block.py:43-57) against the CPU oracle on the same seeded
parameters and inputs, forward and backward.

Tolerances: RoPE and the norms compute in fp32 like the oracle: 1e-5 relative (the only differences
are the sin/cos and rsqrt implementations and summation order). Attention and the block compute their
GEMMs and attention in bf16 with fp32 accumulation: outputs within 1e-2 relative, gradients within 5e-2.
"""
import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200.model import (Attention, HybridElasticNorm, L2Norm, QKNorm, RMSNorm, RotaryEmbedding,
                             TransformerBlock, functional_l2_norm, functional_rms_norm)
from rgpt_b200.model.config import Config
from rgpt_b200.model.norm import ElasticBallNorm, HyperballNorm

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _leaf(t, dev=None):
    return t.detach().clone().to(dev if dev is not None else t.device).requires_grad_(True)


# ------------------------------------------------------------------ RoPE
@pytest.mark.parametrize("T", [100, 1024])
def test_rotary_embedding_forward_backward(cuda, T):
    B, H, D = 2, 4, 64
    g = torch.Generator().manual_seed(T)
    # q, k as the reference passes them: [B, T, H, D] projections transposed to [B, H, T, D] (strided views)
    q0 = torch.randn(B, T, H, D, generator=g)
    k0 = torch.randn(B, T, H, D, generator=g)
    rope = RotaryEmbedding(D, max_seq_len=2048).to(cuda)
    q = _leaf(q0, cuda)
    k = _leaf(k0, cuda)
    qo, ko = rope(q.transpose(1, 2), k.transpose(1, 2))
    gq, gk = torch.randn(B, H, T, D, generator=g), torch.randn(B, H, T, D, generator=g)
    (qo * gq.to(cuda)).sum().backward(retain_graph=True)
    (ko * gk.to(cuda)).sum().backward()
    qr, kr = _leaf(q0), _leaf(k0)
    cos, sin = O.rope_tables(T, D)
    qro, kro = O.rope_apply(qr.transpose(1, 2), kr.transpose(1, 2), cos, sin)
    ((qro * gq).sum() + (kro * gk).sum()).backward()
    assert qo.shape == (B, H, T, D) and qo.dtype == torch.float32
    assert rel(qo, qro) < 1e-5 and rel(ko, kro) < 1e-5
    assert rel(q.grad, qr.grad) < 1e-5 and rel(k.grad, kr.grad) < 1e-5


def test_rotary_embedding_bf16_input(cuda):
    q = torch.randn(1, 2, 64, 64, device=cuda).bfloat16()
    rope = RotaryEmbedding(64).to(cuda)
    qo, _ = rope(q, q)
    cos, sin = O.rope_tables(64, 64)
    ref, _ = O.rope_apply(q.float().cpu(), q.float().cpu(), cos, sin)
    assert qo.dtype == torch.bfloat16 and rel(qo.float(), ref) < 1e-2


# ------------------------------------------------------------------ norms
NORMS = {
    "rmsnorm": (lambda d: RMSNorm(d, 1e-5), lambda x, m: O.rmsnorm(x, m["weight"], 1e-5)),
    "l2norm": (lambda d: L2Norm(d, 1e-5), lambda x, m: O.l2norm(x, m["temp"], 1e-5)),
    "elastic": (lambda d: HybridElasticNorm(d, eps=1e-5), lambda x, m: O.hybrid_elastic(x, 0.5, 1e-5)),
    "elasticball": (lambda d: ElasticBallNorm(d, eps=1e-5), lambda x, m: O.elastic_ball(x, 0.5, 1e-5)),
    "hyperball": (lambda d: HyperballNorm(), lambda x, m: O.hyperball(x)),
}


@pytest.mark.parametrize("d", [64, 100, 512])
@pytest.mark.parametrize("name", list(NORMS))
def test_norm_module_any_dim(cuda, name, d):
    make, ref_fn = NORMS[name]
    torch.manual_seed(d)
    mod = make(d)
    with torch.no_grad():  # non-trivial learned parameters
        for p in mod.parameters():
            p.add_(0.3 * torch.randn_like(p))
    x0 = torch.randn(3, 37, d) * 1.7
    gy = torch.randn(3, 37, d)
    mod_c = mod.to(cuda)
    x = _leaf(x0, cuda)
    y = mod_c(x)
    (y * gy.to(cuda)).sum().backward()
    xr = _leaf(x0)
    params = {k: _leaf(v.cpu()) for k, v in mod.named_parameters()}
    yr = ref_fn(xr, params)
    (yr * gy).sum().backward()
    assert y.shape == x0.shape and y.dtype == torch.float32
    assert rel(y, yr) < 1e-5, rel(y, yr)
    assert rel(x.grad, xr.grad) < 1e-5, rel(x.grad, xr.grad)
    for k, p in mod_c.named_parameters():
        assert rel(p.grad, params[k].grad) < 1e-5, (k, rel(p.grad, params[k].grad))


@pytest.mark.parametrize("fn", ["f_rmsnorm", "f_l2norm"])
def test_functional_norms(cuda, fn):
    # a random upstream gradient: the squared norm of a normalised row is constant, its gradient zero
    x0, gy = torch.randn(50, 64) * 3, torch.randn(50, 64)
    x = _leaf(x0, cuda)
    y = functional_rms_norm(x, 1e-5) if fn == "f_rmsnorm" else functional_l2_norm(x, 1e-5)
    (y * gy.to(cuda)).sum().backward()
    xr = _leaf(x0)
    yr = O.f_rmsnorm(xr) if fn == "f_rmsnorm" else O.f_l2norm(xr, 1e-5)
    (yr * gy).sum().backward()
    assert rel(y, yr) < 1e-5 and rel(x.grad, xr.grad) < 1e-5


QK_TYPES = ["f_rmsnorm", "rmsnorm", "l2norm", "f_l2norm", "elastic", "elasticball", "dual_elasticball",
            "hyperball", "asymmetric_hyperball", "identity"]


@pytest.mark.parametrize("qk", QK_TYPES)
def test_qknorm_forward(cuda, qk):
    torch.manual_seed(4)
    mod = QKNorm(64, qk, 1e-5)
    with torch.no_grad():
        for p in mod.parameters():
            p.add_(0.2 * torch.randn_like(p))
    state = {k: v.detach().clone() for k, v in mod.state_dict().items()}
    q0, k0 = torch.randn(2, 33, 4, 64), torch.randn(2, 33, 4, 64)
    gq, gk = torch.randn(2, 33, 4, 64), torch.randn(2, 33, 4, 64)
    mod = mod.to(cuda)
    q, k = _leaf(q0, cuda), _leaf(k0, cuda)
    qo, ko = mod(q, k)
    ((qo * gq.to(cuda)).sum() + (ko * gk.to(cuda)).sum()).backward()
    params = {f"qk.{n}": _leaf(v) for n, v in state.items() if v.is_floating_point() and v.dim() > 0
              and not n.endswith(("eps", "scale_q", "scale_k"))}
    qr, kr = _leaf(q0), _leaf(k0)
    qro, kro = O.qk_norm_apply(qk, qr, kr, params, "qk", 1e-5, 64)
    ((qro * gq).sum() + (kro * gk).sum()).backward()
    assert rel(qo, qro) < 1e-5 and rel(ko, kro) < 1e-5
    assert rel(q.grad, qr.grad) < 1e-5 and rel(k.grad, kr.grad) < 1e-5
    for n, p in mod.named_parameters():
        assert rel(p.grad, params[f"qk.{n}"].grad) < 1e-5, n


# ------------------------------------------------------------------ attention / block
BASE = dict(name="gpt", n_layers=2, n_recur=1, detach_recur=False, cal_halt_loss=False, n_heads=2, d_model=128,
            vocab_size=384, max_seq_len=256, dropout=0.0, norm_type="rmsnorm", norm_eps=1e-5,
            qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=True,
            pad_token_id=-100, tie_word_embeddings=False)


def _randomise(mod, seed):
    torch.manual_seed(seed)
    with torch.no_grad():
        for n, p in mod.named_parameters():
            if p.dim() == 1:  # norm weights, temperatures, biases, layer scales away from their init
                p.add_(0.2 * torch.randn_like(p))


@pytest.mark.parametrize("qk,gate", [("f_rmsnorm", True), ("rmsnorm", True), ("l2norm", False),
                                     ("dual_elasticball", True), ("asymmetric_hyperball", False)])
def test_attention_forward_backward(cuda, qk, gate):
    cfg = dict(BASE, qk_normtype=qk, g1_gate=gate)
    torch.manual_seed(1)
    attn = Attention(Config(cfg))
    _randomise(attn, 2)
    state = {f"a.{k}": v.detach().clone() for k, v in attn.state_dict().items()}
    x0 = torch.randn(2, 100, 128)
    gy = torch.randn(2, 100, 128)
    attn = attn.to(cuda).train()
    x = _leaf(x0, cuda)
    y = attn(x)
    (y * gy.to(cuda)).sum().backward()
    params = {k: _leaf(v) for k, v in state.items() if v.is_floating_point() and not k.endswith(
        ("inv_freq", "eps", "scale_q", "scale_k"))}
    xr = _leaf(x0)
    yr = O.attention_forward(xr, params, "a", cfg)
    (yr * gy).sum().backward()
    assert y.shape == x0.shape and y.dtype == torch.float32
    assert rel(y, yr) < 1e-2, rel(y, yr)
    assert rel(x.grad, xr.grad) < 5e-2, rel(x.grad, xr.grad)
    for n, p in attn.named_parameters():
        gr = params[f"a.{n}"].grad
        if gr is None or gr.abs().max() == 0:
            continue
        assert rel(p.grad, gr) < 5e-2, (n, rel(p.grad, gr))


def test_attention_forward_with_dropout(cuda):
    """Training-mode Attention draws its probability dropout from its own Philox key; the oracle
    regenerates the same mask (site 2 of that key) and must agree."""
    cfg = dict(BASE, dropout=0.1)
    torch.manual_seed(5)
    attn = Attention(Config(cfg))
    state = {f"a.{k}": v.detach().clone() for k, v in attn.state_dict().items()}
    x0 = torch.randn(2, 64, 128)
    attn = attn.to(cuda).train()
    x = _leaf(x0, cuda)
    y = attn(x)
    seed = int(attn._seed.item())
    y.square().sum().backward()
    params = {k: _leaf(v) for k, v in state.items() if v.is_floating_point() and not k.endswith(("inv_freq",))}
    xr = _leaf(x0)
    yr = O.attention_forward(xr, params, "a", cfg, drop={"p": 0.1, "seed": seed, "site": 0})
    yr.square().sum().backward()
    y_nodrop = O.attention_forward(x0, {k: v.detach() for k, v in params.items()}, "a", cfg)
    assert rel(y_nodrop, yr) > 1e-2  # the mask is in effect
    assert rel(y, yr) < 1e-2 and rel(x.grad, xr.grad) < 5e-2
    with torch.no_grad():  # eval mode: no dropout
        ye = attn.eval()(x0.to(cuda))
    assert rel(ye, y_nodrop) < 1e-2


@pytest.mark.parametrize("norm_type,ls", [("rmsnorm", True), ("l2norm", False), ("f_rmsnorm", True)])
def test_transformer_block_forward_backward(cuda, norm_type, ls):
    cfg = dict(BASE, norm_type=norm_type, use_layer_scale=ls, activation_type="gelu")
    torch.manual_seed(3)
    blk = TransformerBlock(Config(cfg))
    _randomise(blk, 4)
    state = {f"b.{k}": v.detach().clone() for k, v in blk.state_dict().items()}
    x0 = torch.randn(2, 100, 128)
    gy = torch.randn(2, 100, 128)
    blk = blk.to(cuda).train()
    x = _leaf(x0, cuda)
    y = blk(x)
    (y * gy.to(cuda)).sum().backward()
    params = {k: _leaf(v) for k, v in state.items() if v.is_floating_point() and not k.endswith(
        ("inv_freq", "eps", "scale_q", "scale_k"))}
    xr = _leaf(x0)
    yr = O.block_forward(xr, params, "b", cfg)
    (yr * gy).sum().backward()
    assert rel(y, yr) < 1e-2, rel(y, yr)
    assert rel(x.grad, xr.grad) < 5e-2, rel(x.grad, xr.grad)
    for n, p in blk.named_parameters():
        gr = params[f"b.{n}"].grad
        if gr is None or gr.abs().max() == 0:
            continue
        assert rel(p.grad, gr) < 5e-2, (n, rel(p.grad, gr))
