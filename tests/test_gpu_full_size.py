"""The gpt-small and rgpt-small workloads at full model size against the CPU oracle.

Full size means the benchmark's model: d_model 512, 8 heads, vocab 50304, seq 1024, and 8 layers
(gpt-small) or 2 layers x 4 recurrences with halting, layer scale and undetached recurrences
(rgpt-small). Only the micro-batch is cut, to one sequence, so that the fp32 oracle finishes a step
in seconds; rgpt-small accumulates two micro-batches into one optimizer step, as its configuration
accumulates gradients. What only appears at this size is covered here: vocabulary-wide CTA-pair
GEMMs with split-K reduce-adds into the 103 MB lm_head gradient, the 8-layer gradient arena,
T = 1024 attention (with dropout inside a whole step), and 4 recurrences of shared weights
accumulating into one arena.

Tolerances (the bf16 bar of the training step): loss and logits within 1e-2 relative; every
parameter gradient within 5e-2 relative Frobenius error; one optimizer step on identical gradients:
AdamW updates within 1e-4, Muon updates within 5e-2 (bf16 Newton-Schulz rounding; the reference's own
bf16 and fp32 iterations differ by 2.3 %). With dropout the oracle regenerates the kernels' Philox
masks from the step's seed.
"""
import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200.model import GPT
from rgpt_b200.optimizer import Muon, trainer_param_groups
from rgpt_b200.workloads import OPT, WORKLOADS

pytestmark = pytest.mark.gpu

SKIP = (".eps", "inv_freq", "scale_q", "scale_k")


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _setup(name, dropout, seed):
    wl = WORKLOADS[name]
    cfg = dict(wl["cfg"], dropout=dropout)
    torch.manual_seed(seed)
    model = GPT(**cfg)
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    return cfg, wl["T"], model, state


def _oracle_params(state, grad=True):
    return {k: v.clone().requires_grad_(grad) for k, v in state.items() if v.is_floating_point() and not k.endswith(SKIP)}


@pytest.mark.parametrize("dropout", [0.0, 0.1], ids=["p0", "p0.1"])
@pytest.mark.parametrize("name", ["gpt-small", "rgpt-small"])
def test_full_size_training_step_matches_oracle(cuda, name, dropout):
    cfg, T, model, state = _setup(name, dropout, seed=11)
    micro = 2 if name == "rgpt-small" else 1
    g = torch.Generator().manual_seed(12)
    ids = torch.randint(0, cfg["vocab_size"], (micro, 1, T + 1), generator=g)
    labels = ids.clone()
    labels[:, 0, 5] = -100  # an ignored position (pad_token_id = -100)
    model = model.to(cuda).train()
    opt = Muon(trainer_param_groups(model), **OPT)
    opt.zero_grad(set_to_none=True)
    ours, seeds = [], []
    for a in range(micro):
        total, _, _ = model.forward_loss(ids[a, :, :-1].to(cuda), labels[a, :, 1:].contiguous().to(cuda))
        seeds.append(int(model.engine().drop_seed.item()))
        (total * (1.0 / micro)).backward()
        ours.append(total.item())
    grads = {k: p.grad.detach().cpu().clone() for k, p in model.named_parameters()}
    opt.step()
    torch.cuda.synchronize()
    after = {k: p.detach().cpu().clone() for k, p in model.named_parameters()}

    params = _oracle_params(state)
    for a in range(micro):
        out = O.gpt_forward(params, ids[a, :, :-1], cfg, labels=labels[a, :, 1:].contiguous(), training=True,
                            drop_seed=seeds[a] if dropout > 0 else None)
        loss, _ = O.compute_loss(out, labels[a, :, 1:])
        (loss * (1.0 / micro)).backward()
        assert abs(ours[a] - loss.item()) / loss.item() < 1e-2, (a, ours[a], loss.item())
    for k, p in params.items():
        if p.grad is None or p.grad.abs().max() == 0:
            assert grads[k].abs().max().item() < 1e-6, k
            continue
        assert rel(grads[k], p.grad) < 5e-2, (k, rel(grads[k], p.grad))

    # one Muon + AdamW step from the same gradients
    oparams = _oracle_params(state, grad=False)
    O.OracleMuon(oparams, **OPT).step(grads)
    muon_names, _, _ = O.param_groups(list(oparams.items()))
    for k, p in oparams.items():
        d_ref = p - state[k]
        if d_ref.abs().max() == 0:
            continue
        tol = 5e-2 if k in muon_names else 1e-4
        assert rel(after[k] - state[k], d_ref) < tol, (k, rel(after[k] - state[k], d_ref))


@pytest.mark.parametrize("name", ["gpt-small", "rgpt-small"])
def test_full_size_forward_logits_match_oracle(cuda, name):
    """GPT.forward's logits [1, 1024, 50304] (the reference API) vs the oracle's, eval mode."""
    cfg, T, model, state = _setup(name, 0.1, seed=13)
    ids = torch.randint(0, cfg["vocab_size"], (1, T), generator=torch.Generator().manual_seed(14))
    model = model.to(cuda).eval()
    with torch.no_grad():
        logits, _, _, _ = model(ids.to(cuda))
    ref = O.gpt_forward(_oracle_params(state, grad=False), ids, cfg, training=False)[0]
    assert logits.shape == ref.shape
    assert rel(logits.float(), ref) < 1e-2, rel(logits.float(), ref)
