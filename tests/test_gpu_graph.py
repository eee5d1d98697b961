"""The training step as one CUDA graph (rgpt_b200.graph) and the device-resident optimizer
scalars it relies on.

* Device scalars vs by-value scalars: the same Muon + AdamW updates bit for bit, while the
  learning rate changes every step as a scheduler would change it (trainer.py:108-130).
* Graph replay vs eager steps of a small GPT from the same weights and batches: the same loss
  trajectory and weight updates (to the run-to-run spread of the fp32 atomics in the backward),
  and a learning rate set to 0 between replays leaves every weight bit-identical, i.e. the
  replay reads the scalars staged for that step rather than the ones present at capture.
"""
import copy

import pytest
import torch

from rgpt_b200.graph import GraphedTrainStep
from rgpt_b200.model import GPT
from rgpt_b200.optimizer import Muon, trainer_param_groups

pytestmark = pytest.mark.gpu

CFG = dict(name="gpt", n_layers=2, n_recur=1, detach_recur=False, cal_halt_loss=False, n_heads=2, d_model=128,
           vocab_size=384, max_seq_len=256, dropout=0.0, norm_type="rmsnorm", norm_eps=1e-5,
           qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=False,
           pad_token_id=-100, tie_word_embeddings=False)


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def test_device_scalars_match_by_value_bitwise(cuda):
    g = torch.Generator().manual_seed(11)
    w0 = torch.randn(48, 64, generator=g) * 0.02  # one 64x64 tile: the norm reduction has a fixed order
    b0 = torch.randn(64, generator=g)
    grads = [(torch.randn(48, 64, generator=g) * 1e-2, torch.randn(64, generator=g) * 1e-3) for _ in range(3)]
    sides = []
    for device_scalars in (False, True):
        W = torch.nn.Parameter(w0.clone().to(cuda))
        Bv = torch.nn.Parameter(b0.clone().to(cuda))
        opt = Muon([{"params": [W], "use_muon": True}, {"params": [Bv], "use_muon": False, "weight_decay": 0.1}],
                   lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
        if device_scalars:
            opt.use_device_hparams()
        for i, (gw, gb) in enumerate(grads):
            for group in opt.param_groups:
                group["lr"] = 6e-4 * (1.0 + 0.5 * i)  # a scheduler's per-step learning rate
            opt.param_groups[0]["momentum"] = 0.95 - 0.01 * i  # and momentum (OneCycleLR cycles it)
            W.grad, Bv.grad = gw.to(cuda), gb.to(cuda)
            if device_scalars:
                opt.stage_device_hparams()
            opt.step()
        torch.cuda.synchronize()
        sides.append((W.detach().cpu(), Bv.detach().cpu(), opt.state[W]["momentum_buffer"].cpu(),
                      opt.state[Bv]["exp_avg"].cpu(), opt.state[Bv]["exp_avg_sq"].cpu(),
                      opt.param_groups[1]["_adam_step"]))
    for a, b in zip(*sides):
        if isinstance(a, int):
            assert a == b == 3
        else:
            assert torch.equal(a, b)
    assert not torch.equal(sides[0][0], w0)


def _eager_step(model, opt, ids):
    opt.zero_grad(set_to_none=True)
    total, _, _ = model.forward_loss(ids[0, :, :-1], ids[0, :, 1:])
    total.backward()
    opt.step()
    return total


def test_graphed_step_matches_eager_and_reads_staged_scalars(cuda):
    torch.manual_seed(0)
    base = GPT(**CFG)
    B, T = 2, 128
    g = torch.Generator().manual_seed(1)
    batches = [torch.randint(0, CFG["vocab_size"], (1, B, T + 1), generator=g).pin_memory() for _ in range(5)]
    w0 = {k: v.detach().clone() for k, v in base.state_dict().items()}

    m_e = copy.deepcopy(base).to(cuda).train()
    o_e = Muon(trainer_param_groups(m_e), lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    m_g = copy.deepcopy(base).to(cuda).train()
    o_g = Muon(trainer_param_groups(m_g), lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    step = GraphedTrainStep(m_g, o_g, B, T, accum=1, warmup=1)

    losses_e, losses_g = [], []
    for ids in batches:
        losses_e.append(_eager_step(m_e, o_e, ids.to(cuda)).item())
        losses_g.append(step(ids).item())
    assert step.graph is not None and step.launches > 50
    for a, b in zip(losses_e, losses_g):
        assert abs(a - b) <= 1e-3 * abs(a), (losses_e, losses_g)
    pe, pg = dict(m_e.named_parameters()), dict(m_g.named_parameters())
    for k, p in pg.items():
        d_g = p.detach().cpu() - w0[k]
        d_e = pe[k].detach().cpu() - w0[k]
        if d_e.abs().max() == 0:
            continue
        assert rel(d_g, d_e) < 5e-2, (k, rel(d_g, d_e))
    assert o_g.param_groups[1]["_adam_step"] == len(batches)

    # learning rate 0 from here on: the next replay must leave every weight bit-identical
    before = {k: p.detach().clone() for k, p in pg.items()}
    for group in o_g.param_groups:
        group["lr"] = 0.0
    step(batches[0])
    torch.cuda.synchronize()
    for k, p in pg.items():
        assert torch.equal(p.detach(), before[k]), k
