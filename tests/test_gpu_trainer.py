"""The Trainer (trainer.py:19-322) on the native path: resume, validation, multiple-choice test, data loader.

1. Resume: 3 steps (cosine schedule with warm-up, 2 accumulated micro-batches each), save_checkpoint,
   a fresh model and Trainer load_checkpoint, 2 more steps; the result must equal 5 uninterrupted
   steps. Loading restores parameters, optimizer state (bf16 momentum included) and the learning rates
   exactly; the continued run agrees within 1e-2 relative on the parameter updates (the split-K fp32
   atomics of the weight gradients sum in a varying order, and Muon's bf16 Newton-Schulz amplifies the
   last-bit differences).
2. Validation on {"src", "tgt"} batches and test on multiple-choice {"input_ids", "labels", ...}
   batches (the schema the reference's _validate_loss cannot read): losses within 1e-2 of the oracle's,
   and the multiple-choice accuracy equal to the oracle's choice wherever the oracle's best ending
   wins by more than 1 %.
3. train() end to end on a ShardLoader over a token shard (pinned prefetch, side-stream copies).
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import ref_ops as O
from rgpt_b200.data import ShardLoader, hellaswag_collate_fn, write_token_shard
from rgpt_b200.model import GPT
from rgpt_b200.trainer import Trainer

pytestmark = pytest.mark.gpu

MODEL = dict(name="rgpt", n_layers=1, n_recur=2, detach_recur=False, cal_halt_loss=True, n_heads=2, d_model=128,
             vocab_size=384, max_seq_len=256, dropout=0.0, norm_type="rmsnorm", norm_eps=1e-5,
             qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=True,
             pad_token_id=-100, tie_word_embeddings=False)


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def make_cfg(out_dir, total_steps=5, **training):
    t = dict(grad_accum_steps=2, total_steps=total_steps, early_stopping_patience=-1, val_every_n_steps=1000,
             optimizer=dict(lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3),
             scheduler=dict(name="cosine", warmup_steps=2))
    t.update(training)
    return {"model": dict(MODEL), "training": t, "output_dir": str(out_dir)}


def trainer_for(cfg, seed, cuda, **loaders):
    torch.manual_seed(seed)
    model = GPT(**cfg["model"])
    return Trainer(cfg, model, loaders.get("train"), loaders.get("val"), loaders.get("test"), cuda, 0, 1)


def batches(n_steps, accum, B=2, T=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n_steps):
        micro = []
        for _ in range(accum):
            ids = torch.randint(0, MODEL["vocab_size"], (B, T + 1), generator=g)
            micro.append((ids, ids))
        out.append(micro)
    return out


def test_checkpoint_resume_matches_uninterrupted(cuda, tmp_path):
    data = batches(5, 2)
    ta = trainer_for(make_cfg(tmp_path / "a"), 0, cuda)
    init = {k: v.detach().clone() for k, v in ta.model.state_dict().items()}
    for micro in data:
        ta.train_step(micro)
    final_a = {k: v.detach().clone() for k, v in ta.model.state_dict().items()}

    tb = trainer_for(make_cfg(tmp_path / "b"), 0, cuda)
    for micro in data[:3]:
        tb.train_step(micro)
    path = tmp_path / "ck.pth"
    tb.save_checkpoint(path, tb.global_step)
    saved_params = {k: v.detach().clone() for k, v in tb.model.state_dict().items()}
    names_b = {p: n for n, p in tb.model.named_parameters()}
    saved_state = {names_b[p]: {k: v.clone() for k, v in st.items() if torch.is_tensor(v)}
                   for p, st in tb.optimizer.state.items()}
    saved_lrs = [g["lr"] for g in tb.optimizer.param_groups]

    tc = trainer_for(make_cfg(tmp_path / "c"), 123, cuda)  # different init: the load must overwrite it
    tc.train_step(data[0])  # creates optimizer state (and its descriptor tables) before the load
    tc.load_checkpoint(path)
    assert tc.global_step == 3
    for k, v in tc.model.state_dict().items():
        assert torch.equal(v, saved_params[k]), k
    names_c = {p: n for n, p in tc.model.named_parameters()}
    assert {names_c[p] for p in tc.optimizer.state} == set(saved_state)
    for p, st in tc.optimizer.state.items():
        for k, v in saved_state[names_c[p]].items():
            assert st[k].dtype == v.dtype and torch.equal(st[k], v), (names_c[p], k)
    assert [g["lr"] for g in tc.optimizer.param_groups] == saved_lrs
    for micro in data[3:]:
        tc.train_step(micro)
    assert [g["lr"] for g in tc.optimizer.param_groups] == [g["lr"] for g in ta.optimizer.param_groups]
    for k, v in tc.model.state_dict().items():
        if not v.is_floating_point() or k.endswith(("eps", "inv_freq")):
            continue
        d_ref = final_a[k] - init[k]
        if d_ref.abs().max() == 0:
            assert torch.equal(v, final_a[k]), k
            continue
        assert rel(v - init[k], d_ref) < 1e-2, (k, rel(v - init[k], d_ref))


class ToyTokenizer:
    pad_token_id = None
    eos_token_id = 1
    bos_token_id = 2

    def encode(self, text, add_special_tokens=True):
        return [3 + (ord(c) % 97) for c in text]


MC_ITEMS = [{"context": f"item {i}: " + "ab" * (i % 5), "endings": [f"end {j} " * (1 + (i + j) % 3) for j in range(4)],
             "label": i % 4} for i in range(12)]


def oracle_token_losses(state, cfg, ids, labels):
    params = {k: v for k, v in state.items() if v.is_floating_point() and not k.endswith((".eps", "inv_freq"))}
    logits = O.gpt_forward(params, ids[:, :-1], cfg, training=False)[0]
    lab = labels[:, 1:]
    return F.cross_entropy(logits.reshape(-1, logits.size(-1)), lab.reshape(-1), ignore_index=-100,
                           reduction="none").view(lab.shape), lab


def test_validation_and_multiple_choice_test(cuda, tmp_path):
    g = torch.Generator().manual_seed(3)
    val = [{"src": ids, "tgt": ids} for ids in torch.randint(0, MODEL["vocab_size"], (3, 2, 65), generator=g)]
    tok = ToyTokenizer()
    test = [hellaswag_collate_fn(MC_ITEMS[i:i + 4], tok, 32) for i in range(0, 12, 4)]
    t = trainer_for(make_cfg(tmp_path), 7, cuda, val=val, test=test)
    state = {k: v.detach().cpu().clone() for k, v in t.model.state_dict().items()}
    cfg = MODEL
    # validation loss: mean over batches of the mean token loss
    ref_val = []
    for b in val:
        tl, lab = oracle_token_losses(state, cfg, b["src"], b["tgt"])
        ref_val.append(tl.sum() / (lab != -100).sum())
    ours_val = t._validate_loss(val)
    assert abs(ours_val - torch.stack(ref_val).mean().item()) / torch.stack(ref_val).mean().item() < 1e-2
    # multiple-choice test: loss and accuracy
    loss = t.test()
    ref_loss, agree, correct_sum, correct_mean, n_items = [], 0, 0, 0, 0
    for b in test:
        tl, lab = oracle_token_losses(state, cfg, b["input_ids"], b["labels"])
        ref_loss.append(tl.sum() / (lab != -100).sum())
        tot = tl.sum(1)
        mean = tot / (lab != -100).sum(1).clamp_min(1)
        for i in range(int(b["correct_labels"].numel())):
            rows = (b["example_indices"] == i).nonzero().flatten()
            s = tot[rows]
            best = int(torch.argmin(s))
            gap = (s.sort().values[1] - s.min()) / s.min().abs()
            correct_sum += int(best == int(b["correct_labels"][i]))
            correct_mean += int(int(torch.argmin(mean[rows])) == int(b["correct_labels"][i]))
            n_items += 1
            agree += int(gap > 1e-2)
    assert abs(loss - torch.stack(ref_loss).mean().item()) / torch.stack(ref_loss).mean().item() < 1e-2
    m = t.test_metrics
    assert n_items == 12 and "Acc/test" in m
    # the native per-token losses pick the oracle's ending (near-ties within 1 % aside)
    assert abs(m["Acc/test"] * 12 - correct_sum) <= 12 - agree
    assert abs(m["Acc/test_norm"] * 12 - correct_mean) <= 12 - agree


def test_train_loop_on_shard_loader(cuda, tmp_path):
    path = str(tmp_path / "tokens.bin")
    g = torch.Generator().manual_seed(5)
    write_token_shard(path, [torch.randint(0, MODEL["vocab_size"], (int(n),), generator=g).tolist()
                             for n in torch.randint(50, 500, (40,), generator=g)], MODEL["vocab_size"])
    train = ShardLoader(path, 2, 65, device=cuda, seed=1)
    val = ShardLoader(path, 2, 65, device=cuda, shuffle=False)
    cfg = make_cfg(tmp_path / "out", total_steps=4, val_every_n_steps=2)
    t = trainer_for(cfg, 11, cuda, train=train, val=val)
    t.train()
    assert t.global_step == 4
    assert t.best_metric < float("inf") and t.best_model_path.exists()
    ck = torch.load(t.best_model_path, weights_only=False)
    assert set(ck) >= {"model_state_dict", "optimizer_state_dict", "best_metric", "global_step"}
