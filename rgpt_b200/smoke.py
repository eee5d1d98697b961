"""One tiny native training step on cuda:0 checked against the CPU oracle.

The step is an rGPT one (recurrence, halting loss, layer scale) with dropout 0.1, the reference
configs' rate; the oracle regenerates the kernels' dropout masks from the same seed.

The oracle is imported here only as the checker (this module backs
__graft_entry__.smoke()); the step itself runs the native kernels."""
import torch


def run_smoke() -> None:
    from oracle import ref_ops as O

    from .model import GPT
    from .optimizer import Muon, trainer_param_groups

    cfg = dict(name="rgpt", n_layers=1, n_recur=2, detach_recur=False, cal_halt_loss=True, n_heads=2, d_model=128,
               vocab_size=384, max_seq_len=128, dropout=0.1, norm_type="rmsnorm", norm_eps=1e-5,
               qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=True,
               pad_token_id=-100, tie_word_embeddings=False)
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    model = GPT(**cfg)
    state = {k: v.detach().clone() for k, v in model.state_dict().items()}
    ids = torch.randint(0, cfg["vocab_size"], (2, 129), generator=torch.Generator().manual_seed(1))
    model = model.to(dev).train()
    opt = Muon(trainer_param_groups(model), lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    total, tok, q = model.forward_loss(ids[:, :-1].to(dev), ids[:, 1:].contiguous().to(dev))
    drop_seed = int(model.engine().drop_seed.item())  # the Philox key of this forward's masks
    total.backward()
    g_ours = model.lm_head.weight.grad.detach().cpu().clone()
    opt.step()
    torch.cuda.synchronize()

    params = {k: v.clone().requires_grad_(True) for k, v in state.items()
              if v.is_floating_point() and not k.endswith((".eps", "inv_freq"))}
    out = O.gpt_forward(params, ids[:, :-1], cfg, labels=ids[:, 1:].contiguous(), training=True,
                        drop_seed=drop_seed)
    ref_loss, _ = O.compute_loss(out, ids[:, 1:])
    ref_loss.backward()
    lrel = abs(total.item() - ref_loss.item()) / abs(ref_loss.item())
    g_ref = params["lm_head.weight"].grad
    grel = ((g_ours - g_ref).norm() / g_ref.norm()).item()
    if not (lrel < 1e-2 and grel < 5e-2):
        raise RuntimeError(f"smoke mismatch: loss rel {lrel:.3e}, lm_head grad rel {grel:.3e}")
    print(f"smoke ok: loss {total.item():.5f} (oracle {ref_loss.item():.5f}), lm_head grad rel err {grel:.2e}")
