"""Full GPT / rGPT training step on the native engine vs the CPU oracle.

The oracle (oracle/ref_ops.py, pinned to the reference by tests/golden) runs the
same seeded parameters and tokens in fp32 on the CPU. The native path computes
in bf16 with fp32 accumulation and an fp32 residual stream.

Tolerances: loss and logits within 1e-2 relative (the bf16 bar); per-parameter
gradients within 5e-2 relative Frobenius error (bf16 operands through up to
~20 chained GEMMs / attention); one optimizer step: AdamW updates within 1e-4,
Muon updates within 5e-2 (bf16 Newton-Schulz rounding).
"""
import copy

import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200.model import GPT
from rgpt_b200.optimizer import Muon, trainer_param_groups

pytestmark = pytest.mark.gpu

BASE = dict(name="gpt", n_layers=2, n_recur=1, detach_recur=False, cal_halt_loss=False, n_heads=2, d_model=128,
            vocab_size=384, max_seq_len=256, dropout=0.0, norm_type="rmsnorm", norm_eps=1e-5,
            qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=False,
            pad_token_id=-100, tie_word_embeddings=False)
CFGS = {
    "gpt": BASE,
    "rgpt": dict(BASE, name="rgpt", n_layers=1, n_recur=3, cal_halt_loss=True, use_layer_scale=True),
    "rgpt_detach": dict(BASE, name="rgpt", n_layers=2, n_recur=2, cal_halt_loss=True, use_layer_scale=True,
                        detach_recur=True),
    "elastic_gelu": dict(BASE, qk_normtype="elastic", use_layer_scale=True, activation_type="gelu"),
    "qk_rmsnorm": dict(BASE, qk_normtype="rmsnorm", use_layer_scale=True),
    "asym_hyperball_silu": dict(BASE, qk_normtype="asymmetric_hyperball", activation_type="silu"),
    "dual_elasticball_mish": dict(BASE, qk_normtype="dual_elasticball", activation_type="mish"),
    "no_qk": dict(BASE, qk_normtype="identity"),
    "elasticball": dict(BASE, qk_normtype="elasticball", use_layer_scale=True),
    "hyperball": dict(BASE, qk_normtype="hyperball", use_layer_scale=True),
    # residual-stream norm kinds other than rmsnorm (model/norm.py:37-95): L2Norm with its learned
    # temperature (and gradient), the functional L2 and RMS norms, the hybrid elastic norm
    "resid_l2norm": dict(BASE, norm_type="l2norm", use_layer_scale=True),
    "resid_f_l2norm": dict(BASE, norm_type="f_l2norm"),
    "resid_f_rmsnorm": dict(BASE, norm_type="f_rmsnorm", qk_normtype="l2norm"),
    "resid_elastic_rgpt": dict(BASE, name="rgpt", n_layers=1, n_recur=2, cal_halt_loss=True, use_layer_scale=True,
                               norm_type="elastic"),
}


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def make(tag, seed=0, B=2, T=128):
    cfg = CFGS[tag]
    torch.manual_seed(seed)
    model = GPT(**cfg)
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    g = torch.Generator().manual_seed(seed + 1)
    ids = torch.randint(0, cfg["vocab_size"], (B, T + 1), generator=g)
    labels = ids.clone()
    labels[0, 7] = -100
    return cfg, model, state, ids, labels


def oracle_step(cfg, state, ids, labels):
    params = {k: v.clone().requires_grad_(True) for k, v in state.items()
              if v.is_floating_point() and not k.endswith((".eps", "inv_freq", "scale_q", "scale_k"))}
    out = O.gpt_forward(params, ids[:, :-1], cfg, labels=labels[:, 1:].contiguous(), training=True)
    loss, tok = O.compute_loss(out, labels[:, 1:])
    loss.backward()
    return loss.item(), out[0].detach(), {k: p.grad for k, p in params.items() if p.grad is not None}


@pytest.mark.parametrize("tag", list(CFGS))
def test_fused_loss_and_grads_match_oracle(cuda, tag):
    cfg, model, state, ids, labels = make(tag)
    model = model.to(cuda).train()
    total, tok, q = model.forward_loss(ids[:, :-1].to(cuda), labels[:, 1:].contiguous().to(cuda))
    total.backward()
    torch.cuda.synchronize()
    ref_loss, _, ref_grads = oracle_step(cfg, state, ids, labels)
    assert abs(total.item() - ref_loss) / abs(ref_loss) < 1e-2, (total.item(), ref_loss)
    named = dict(model.named_parameters())
    for k, gref in ref_grads.items():
        if gref.abs().max() == 0:
            assert named[k].grad.abs().max().item() < 1e-6, k
            continue
        assert rel(named[k].grad, gref) < 5e-2, (k, rel(named[k].grad, gref))


@pytest.mark.parametrize("tag", ["gpt", "rgpt"])
def test_api_forward_logits_and_autograd(cuda, tag):
    import torch.nn.functional as F
    cfg, model, state, ids, labels = make(tag, seed=3)
    model = model.to(cuda).train()
    inp, tgt = ids[:, :-1].to(cuda), labels[:, 1:].contiguous().to(cuda)
    logits, halt, qs, targets = model(inp, labels=tgt)
    ref_loss, ref_logits, ref_grads = oracle_step(cfg, state, ids, labels)
    assert rel(logits.float(), ref_logits) < 1e-2
    # reference-style loss on the returned outputs (trainer.py:139-167)
    loss = F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), tgt.reshape(-1), ignore_index=-100)
    if cfg["cal_halt_loss"]:
        qc = sum(F.binary_cross_entropy_with_logits(qs[i][..., 1], targets[i]) for i in range(len(qs))) / len(qs)
        loss = loss + qc + halt / len(qs)
    loss.backward()
    assert abs(loss.item() - ref_loss) / ref_loss < 1e-2
    named = dict(model.named_parameters())
    for k in ("lm_head.weight", "layers.0.attn.q_proj.weight", "layers.0.ff.fc1.weight", "embs.weight"):
        assert rel(named[k].grad, ref_grads[k]) < 5e-2, k


def test_eval_forward_logits(cuda):
    cfg, model, state, ids, labels = make("gpt", seed=5)
    model = model.to(cuda).eval()
    with torch.no_grad():
        logits, _, _, _ = model(ids[:, :-1].to(cuda))
    _, ref_logits, _ = oracle_step(cfg, state, ids, labels)
    assert rel(logits.float(), ref_logits) < 1e-2


def test_muon_adamw_step_matches_oracle(cuda):
    cfg, model, state, ids, labels = make("rgpt", seed=7)
    model = model.to(cuda).train()
    opt = Muon(trainer_param_groups(model), lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    total, _, _ = model.forward_loss(ids[:, :-1].to(cuda), labels[:, 1:].contiguous().to(cuda))
    total.backward()
    grads = {k: p.grad.detach().cpu().clone() for k, p in model.named_parameters()}
    opt.step()
    torch.cuda.synchronize()
    params = {k: v.clone() for k, v in state.items() if v.is_floating_point()
              and not k.endswith((".eps", "inv_freq"))}
    oopt = O.OracleMuon(params, lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    oopt.step({k: g for k, g in grads.items()})
    named = dict(model.named_parameters())
    muon_names, _, _ = O.param_groups(list(model.named_parameters()))
    for k, p in params.items():
        d_ours = named[k].detach().cpu() - state[k]
        d_ref = p - state[k]
        if d_ref.abs().max() == 0:
            continue
        # Both sides get identical gradients here. AdamW is plain fp32 arithmetic (1e-4). Muon goes
        # through 15 bf16 GEMMs whose fused epilogues round once where the reference rounds after
        # every op; the reference's own bf16 vs fp32 Newton-Schulz differ by ~2.3%, so 5e-2.
        tol = 5e-2 if k in muon_names else 1e-4
        assert rel(d_ours, d_ref) < tol, (k, rel(d_ours, d_ref))
    # the bf16 shadow the GEMMs read was refreshed by the optimizer kernels
    w = named["layers.0.attn.q_proj.weight"]
    assert rel(w._rgpt_shadow.float(), w.detach().float()) < 1e-2


def test_training_loss_curve_tracks_oracle(cuda):
    cfg, model, state, ids, labels = make("gpt", seed=9, T=128)
    model = model.to(cuda).train()
    opt = Muon(trainer_param_groups(model), lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    # a repeated batch the model can memorise, so the curve really moves (from ~ln V downwards)
    g = torch.Generator().manual_seed(123)
    batches = [torch.randint(0, cfg["vocab_size"], (2, 129), generator=g)] * 8
    ours = []
    for b in batches:
        opt.zero_grad(set_to_none=True)
        total, _, _ = model.forward_loss(b[:, :-1].to(cuda), b[:, 1:].contiguous().to(cuda))
        total.backward()
        opt.step()
        ours.append(total.item())
    params = {k: v for k, v in state.items() if v.is_floating_point() and not k.endswith((".eps", "inv_freq"))}
    ref, _ = O.train_steps(params, cfg, iter([[(b, b)] for b in batches]), len(batches),
                           opt_kwargs=dict(lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3))
    assert ref[-1] < 0.8 * ref[0], ref  # the oracle learned; ours must follow the same curve
    for a, r in zip(ours, ref):
        assert abs(a - r) / r < 2e-2, (ours, ref)


def test_loss_curve_tracks_oracle_over_200_steps(cuda):
    """200 optimizer steps (Muon + AdamW, the Trainer's groups and hyper-parameters) on the native
    engine vs the fp32 CPU oracle from the same seeded weights and batches. Each step draws 2 of 12
    fixed sequences, so the curve keeps moving for all 200 steps (5.2 -> 0.2). bf16 compute makes the
    trajectories drift apart slowly, and the order of the fp32 atomic adds in the split-K weight
    gradients varies from run to run; each 20-step window's mean loss must agree to 2 % + 0.01
    (measured on a B200: 0.0005 to 0.005 apart in the last window, whose loss is ~0.21)."""
    cfg, model, state, _, _ = make("gpt", seed=21, T=64)
    model = model.to(cuda).train()
    kw = dict(lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    opt = Muon(trainer_param_groups(model), **kw)
    g = torch.Generator().manual_seed(77)
    pool = torch.randint(0, cfg["vocab_size"], (12, 65), generator=g)
    picks = [torch.randperm(12, generator=g)[:2] for _ in range(200)]
    batches = [pool[p] for p in picks]
    ours = []
    for b in batches:
        opt.zero_grad(set_to_none=True)
        total, _, _ = model.forward_loss(b[:, :-1].to(cuda), b[:, 1:].contiguous().to(cuda))
        total.backward()
        opt.step()
        ours.append(total.item())
    params = {k: v for k, v in state.items() if v.is_floating_point() and not k.endswith((".eps", "inv_freq"))}
    ref, _ = O.train_steps(params, cfg, iter([[(b, b)] for b in batches]), len(batches), opt_kwargs=kw)
    ours_t, ref_t = torch.tensor(ours), torch.tensor(ref)
    win_o, win_r = ours_t.view(10, 20).mean(1), ref_t.view(10, 20).mean(1)
    print("native", [round(x, 3) for x in win_o.tolist()])
    print("oracle", [round(x, 3) for x in win_r.tolist()])
    assert win_r[-1] < 0.5 * win_r[0], win_r  # the oracle learned
    dev = (win_o - win_r).abs()
    assert (dev < 2e-2 * win_r + 1e-2).all(), (dev, win_r)
