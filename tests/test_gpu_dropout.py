"""Dropout in the native kernels (nn.Dropout at model/gpt.py:96 and model/transformer_block.py:45,52;
SDPA dropout_p at model/attention.py:57) against the oracle.

torch's own dropout stream cannot be reproduced outside torch, so the native kernels draw their keep
bits from Philox4x32-10 with a documented counter layout, and the oracle (pinned to the published
Philox known-answer vectors) regenerates the same masks. The mask kernels (rgpt_drop_mask, rgpt_attn_drop_mask) draw the bits; the GEMM epilogue and the
attention kernels read them. Checks:
  * every stored mask bit equals the oracle's bit (bit-exact), and the keep rate is ~1 - p;
  * outputs and gradients equal the fp32 reference computed with that mask, at the tolerances of
    the dropout-free tests (1e-2 forward, 2e-2 attention gradients, 5e-2 model gradients);
  * a whole training step with dropout 0.1 matches the oracle step with the same masks.
"""
import math

import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200 import native as nv

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def unpack(words: torch.Tensor) -> torch.Tensor:
    """int32 mask words [..., n] -> bool bits [..., 32 n] (bit j of word w = element 32 w + j)."""
    w = words.cpu().to(torch.int64) & 0xFFFFFFFF
    bits = (w.unsqueeze(-1) >> torch.arange(32)) & 1
    return bits.reshape(*words.shape[:-1], words.shape[-1] * 32).bool()


def seed_tensor(cuda, value):
    return torch.tensor([value], dtype=torch.int64, device=cuda)


@pytest.mark.parametrize("M,N,K,p", [(256, 512, 128, 0.1), (300, 256, 64, 0.35), (4096, 1024, 512, 0.1),
                                     (16384, 512, 2048, 0.1)])  # the last one runs on CTA pairs
def test_resid_gemm_dropout_bits_and_values(cuda, M, N, K, p):
    g = torch.Generator(device=cuda).manual_seed(M + N)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    W = (torch.randn(N, K, device=cuda, generator=g) * 0.1).bfloat16()
    C = torch.randn(M, N, device=cuda, generator=g)
    ls = torch.rand(N, device=cuda, generator=g) + 0.5
    out = torch.empty(M, N, device=cuda)
    raw = torch.empty(M, N, device=cuda)
    mask = torch.full((M, N // 32), -1, device=cuda, dtype=torch.int32)
    seed = 0x1234_5678_9ABC_DEF0 + M
    drop = nv.Drop(mask, seed_tensor(cuda, seed), 7, p)
    nv.drop_mask_rows(drop, M, N)
    nv.gemm(A, W, out, epi=nv.EPI_RESID_F32, c=C, colscale=ls, out2=raw, drop=drop)
    torch.cuda.synchronize()
    keep = O.resid_drop_mask(seed, 7, M, N, p)
    assert torch.equal(unpack(mask), keep)
    assert abs(keep.float().mean().item() - (1 - p)) < 0.02
    acc = A.float() @ W.float().t()
    raw_ref = acc * keep.to(cuda).float() / (1 - p)
    assert rel(raw, raw_ref) < 1e-3
    assert rel(out, C + raw_ref * ls) < 1e-3


def attn_inputs(B, T, H, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    d = H * 64
    qkv = torch.randn(B * T, 3 * d, device=dev, generator=g).bfloat16()
    qk = torch.randn(B * T, 2 * d, device=dev, generator=g).bfloat16()
    gate = torch.sigmoid(torch.randn(B * T, d, device=dev, generator=g)).bfloat16()
    return qk, qkv, gate


@pytest.mark.parametrize("B,T,H,p", [(2, 256, 2, 0.1), (1, 200, 2, 0.3), (2, 1024, 8, 0.1)])
def test_attention_dropout_fwd_bwd(cuda, B, T, H, p):
    d = H * 64
    qk, qkv, gate = attn_inputs(B, T, H, cuda, 11 + T)
    o = torch.empty(B * T, d, device=cuda, dtype=torch.bfloat16)
    og = torch.empty_like(o)
    lse = torch.empty(B, H, T, device=cuda)
    QB = (T + 31) // 32
    mask = torch.zeros(B * H, QB, T, device=cuda, dtype=torch.int32)
    seed, site = 987654321 + T, 4 * 3 + 2
    drop = nv.Drop(mask, seed_tensor(cuda, seed), site, p)
    nv.attn_drop_mask(drop, B, T, H)
    nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H, drop=drop)
    torch.cuda.synchronize()
    keep = O.attn_drop_mask(seed, site, B, H, T, p)                     # [B, H, Tq, Tk]
    # stored words: [bh, q // 32, k], bit q % 32; compare where causal (k <= q < T)
    stored = unpack(mask.transpose(1, 2).contiguous()).view(B, H, T, QB * 32)[..., :T].transpose(-1, -2)
    causal = torch.ones(T, T, dtype=torch.bool).tril()
    assert torch.equal(stored[..., causal], keep[..., causal])
    assert abs(keep[..., causal].float().mean().item() - (1 - p)) < 0.02

    q = qk[:, :d].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    k = qk[:, d:].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    v = qkv[:, 2 * d:].float().view(B, T, H, 64).transpose(1, 2).requires_grad_(True)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(64)
    s = s.masked_fill(~causal.to(cuda), float("-inf"))
    lse_ref = torch.logsumexp(s, dim=-1)
    pr = torch.softmax(s, dim=-1) * keep.to(cuda).float() / (1 - p)
    o_ref = (pr @ v).transpose(1, 2).reshape(B * T, d)
    assert rel(o, o_ref) < 1e-2
    assert rel(og, o_ref * gate.float()) < 1e-2
    assert (lse - lse_ref).abs().max().item() < 1e-3   # the normaliser keeps every probability

    gg = torch.Generator(device=cuda).manual_seed(5)
    dog = torch.randn(B * T, d, device=cuda, generator=gg).bfloat16()
    do = torch.empty_like(o)
    dgp = torch.empty_like(o)
    D = torch.empty(B, H, T, device=cuda)
    dq = torch.empty(B * T, d, device=cuda)
    nv.attn_bwd_prep(dog, o, gate, do, dgp, D, B, T, H, dq_zero=dq)
    dk = torch.empty(B * T, d, device=cuda)
    dqkv = torch.zeros(B * T, 3 * d, device=cuda, dtype=torch.bfloat16)
    nv.attn_bwd(qk, qkv, do, lse, D, dq, dk, dqkv[:, 2 * d:], B, T, H, drop=drop)
    torch.cuda.synchronize()
    (o_ref * gate.float() * dog.float()).sum().backward()
    tok = lambda t: t.transpose(1, 2).reshape(B * T, d)
    assert rel(dq, tok(q.grad)) < 2e-2
    assert rel(dk, tok(k.grad)) < 2e-2
    assert rel(dqkv[:, 2 * d:], tok(v.grad)) < 2e-2


def test_embedding_dropout_fwd_bwd(cuda):
    M, d, V, p = 384, 256, 1000, 0.2
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, V, (M,), generator=g).to(cuda)
    emb = torch.randn(V, d, generator=g).to(cuda)
    x = torch.empty(M, d, device=cuda)
    mask = torch.zeros(M, d // 32, device=cuda, dtype=torch.int32)
    seed = 77
    drop = nv.Drop(mask, seed_tensor(cuda, seed), O.EMB_DROP_SITE, p)
    nv.embedding_fwd(ids, emb, x, drop=drop)
    dx = torch.randn(M, d, generator=g).to(cuda)
    demb = torch.zeros(V, d, device=cuda)
    nv.embedding_bwd(ids, dx, demb, drop=drop)
    torch.cuda.synchronize()
    keep = O.resid_drop_mask(seed, O.EMB_DROP_SITE, M, d, p)
    assert torch.equal(unpack(mask), keep)
    z = keep.to(cuda).float() / (1 - p)
    assert rel(x, emb[ids] * z) < 1e-6
    ref = torch.zeros(V, d, device=cuda).index_add_(0, ids, dx * z)
    assert rel(demb, ref) < 1e-5


BASE = dict(name="gpt", n_layers=2, n_recur=1, detach_recur=False, cal_halt_loss=False, n_heads=2, d_model=128,
            vocab_size=384, max_seq_len=256, dropout=0.1, norm_type="rmsnorm", norm_eps=1e-5,
            qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=False,
            pad_token_id=-100, tie_word_embeddings=False)


@pytest.mark.parametrize("cfg", [BASE, dict(BASE, name="rgpt", n_layers=1, n_recur=3, cal_halt_loss=True,
                                            use_layer_scale=True, dropout=0.2),
                                 # conf/model/rgpt.yaml's combination: detached recurrences + halting
                                 dict(BASE, name="rgpt", n_layers=2, n_recur=2, cal_halt_loss=True,
                                      use_layer_scale=True, detach_recur=True)],
                         ids=["gpt", "rgpt", "rgpt_detach"])
def test_training_step_with_dropout_matches_oracle(cuda, cfg):
    """Loss and every gradient of a dropout training step vs the oracle using the same masks."""
    from rgpt_b200.model import GPT
    torch.manual_seed(0)
    model = GPT(**cfg)
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(1)
    B, T = 2, 128
    ids = torch.randint(0, cfg["vocab_size"], (B, T + 1), generator=g)
    model = model.to(cuda).train()
    total, _, _ = model.forward_loss(ids[:, :-1].to(cuda), ids[:, 1:].contiguous().to(cuda))
    seed = int(model.engine().drop_seed.item())
    total.backward()
    torch.cuda.synchronize()
    params = {k: v.clone().requires_grad_(True) for k, v in state.items()
              if v.is_floating_point() and not k.endswith((".eps", "inv_freq", "scale_q", "scale_k"))}
    out = O.gpt_forward(params, ids[:, :-1], cfg, labels=ids[:, 1:].contiguous(), training=True, drop_seed=seed)
    loss, _ = O.compute_loss(out, ids[:, 1:])
    loss.backward()
    assert abs(total.item() - loss.item()) / loss.item() < 1e-2, (total.item(), loss.item())
    # the same step without dropout gives a visibly different loss: the masks are in effect
    ref_nodrop, _ = O.compute_loss(O.gpt_forward({k: v.detach() for k, v in params.items()}, ids[:, :-1], cfg,
                                                 labels=ids[:, 1:].contiguous(), training=True), ids[:, 1:])
    assert abs(ref_nodrop.item() - loss.item()) > 1e-3
    named = dict(model.named_parameters())
    for k, p in params.items():
        if p.grad is None or p.grad.abs().max() == 0:
            continue
        assert rel(named[k].grad, p.grad) < 5e-2, (k, rel(named[k].grad, p.grad))


def test_eval_mode_has_no_dropout(cuda):
    from rgpt_b200.model import GPT
    torch.manual_seed(0)
    model = GPT(**BASE).to(cuda).eval()
    ids = torch.randint(0, BASE["vocab_size"], (2, 65)).to(cuda)
    s0 = int(model.engine().drop_seed.item())
    with torch.no_grad():
        a = model.forward_loss(ids[:, :-1], ids[:, 1:].contiguous())[0].item()
        b = model.forward_loss(ids[:, :-1], ids[:, 1:].contiguous())[0].item()
    assert a == b and int(model.engine().drop_seed.item()) == s0
