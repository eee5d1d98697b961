"""Trainer with the reference's constructor and methods (trainer.py:19-322).

Same parameter grouping (Muon / AdamW-decay / AdamW-no-decay), LR schedules,
gradient accumulation, validation and checkpoint dictionary as the reference.
The hot loop runs the fused native path (GPT.forward_loss: forward, loss and
in-place dlogits in one pass; loss.backward() runs the native backward), and
reads losses back once per optimizer step instead of twice per micro-batch.

Differences, all on purpose:
  * No DDP wrapper: with world_size > 1 the optimizer is DistMuon, which
    averages gradients over NCCL itself (the reference's DDP all-reduces every
    micro-batch; here it happens once per optimizer step).
  * Compute is bf16 with fp32 accumulation and fp32 master weights whatever
    training.dtype says (no GradScaler needed for bf16).
  * The per-parameter gradient-norm print (one host sync per parameter) is
    opt-in (training.log_grad_norm) and done as one reduction.
  * load_checkpoint() resumes from save_checkpoint()'s dictionary (the
    reference saves but never loads); the dictionary gains the scheduler's
    state under an extra key so a resumed run continues the same schedule.
  * Validation and test batches may use either collate schema: {"src", "tgt"}
    (dataset.py:45-51) or the multiple-choice {"input_ids", "labels", ...}
    (dataset.py:144-149), which the reference's _validate_loss cannot read
    (it looks up batch["src"], trainer.py:278). Multiple-choice batches are
    also scored: accuracy of the ending with the lowest summed loss (acc) and
    with the lowest mean loss per token (acc_norm).
"""
from __future__ import annotations

import math
import os
from pathlib import Path

import torch
import torch.nn.functional as F

from .model.config import as_config
from .optimizer import DistMuon, Muon, trainer_param_groups


def _output_dir(cfg):
    try:
        import hydra  # type: ignore

        return Path(hydra.core.hydra_config.HydraConfig.get().runtime.output_dir)
    except Exception:
        return Path(cfg.get("output_dir", "outputs"))


class _Logger:
    """Rank-0 scalar logger (TensorBoard when available, else a JSON-lines file)."""

    def __init__(self, out_dir: Path, rank: int):
        self.rank = rank
        self.writer = None
        self.fh = None
        if rank != 0:
            return
        out_dir.mkdir(parents=True, exist_ok=True)
        try:
            from torch.utils.tensorboard import SummaryWriter

            self.writer = SummaryWriter(log_dir=str(out_dir))
        except Exception:
            self.fh = open(out_dir / "metrics.jsonl", "a")

    def log(self, metrics: dict, step: int):
        if self.rank != 0:
            return
        if self.writer is not None:
            for k, v in metrics.items():
                self.writer.add_scalar(k, v, step)
        elif self.fh is not None:
            import json

            self.fh.write(json.dumps({"step": step, **metrics}) + "\n")
            self.fh.flush()


class Trainer:
    def __init__(self, cfg, model, train_loader, val_loader, test_loader, device, rank, world_size):
        self.cfg = as_config(cfg) if not hasattr(cfg, "training") else cfg
        self.train_loader, self.val_loader, self.test_loader = train_loader, val_loader, test_loader
        self.device = device
        self.rank, self.world_size = rank, world_size
        self.is_ddp = world_size > 1
        self.is_main_process = rank == 0
        self.model = model.to(device)
        tcfg = self.cfg.training
        get = (lambda c, k, d=None: c.get(k, d)) if hasattr(tcfg, "get") else (lambda c, k, d=None: getattr(c, k, d))
        self.grad_accum_steps = get(tcfg, "grad_accum_steps", 1)
        self.early_stopping_patience = get(tcfg, "early_stopping_patience", 3)
        self.log_grad_norm = bool(get(tcfg, "log_grad_norm", False))
        pad_id = self.cfg.model.get("pad_token_id", -100) if hasattr(self.cfg.model, "get") else -100
        self.pad_id = -100 if pad_id is None else pad_id

        ocfg = tcfg.optimizer
        self.muon_lr_multiplier = get(ocfg, "muon_lr_multiplier", 100.0)
        tie = self.cfg.model.get("tie_word_embeddings", True) if hasattr(self.cfg.model, "get") else True
        groups = trainer_param_groups(self.model, tie_word_embeddings=tie, weight_decay=ocfg.weight_decay)
        opt_cls = DistMuon if self.is_ddp else Muon
        self.optimizer = opt_cls(groups, lr=ocfg.lr, weight_decay=ocfg.weight_decay,
                                 muon_lr_multiplier=self.muon_lr_multiplier)

        scfg = tcfg.scheduler
        name = get(scfg, "name", "linear")
        self.total_steps = tcfg.total_steps
        warmup = get(scfg, "warmup_steps", 1000)
        if name in ("linear", "cosine"):
            from transformers import get_cosine_schedule_with_warmup, get_linear_schedule_with_warmup

            fn = get_linear_schedule_with_warmup if name == "linear" else get_cosine_schedule_with_warmup
            self.scheduler = fn(self.optimizer, warmup, self.total_steps)
        elif name == "onecycle":
            from torch.optim.lr_scheduler import OneCycleLR

            max_lr = get(scfg, "max_lr", 0.01)
            self.scheduler = OneCycleLR(
                self.optimizer,
                max_lr=[max_lr * self.muon_lr_multiplier if g.get("use_muon") else max_lr
                        for g in self.optimizer.param_groups],
                total_steps=self.total_steps, pct_start=get(scfg, "pct_start", 0.3), anneal_strategy="cos")
        else:
            self.scheduler = None
        self.grad_clip = get(tcfg, "grad_clip", None)
        self.output_dir = _output_dir(self.cfg)
        mname = self.cfg.model.get("name", "model") if hasattr(self.cfg.model, "get") else "model"
        self.best_model_path = self.output_dir / f"best_{mname}.pth"
        self.best_metric = float("inf")
        self.best_epoch, self.epochs_no_improve, self.global_step = 0, 0, 0
        self.logger = _Logger(self.output_dir, rank)

    # ------------------------------------------------------------------ losses
    def compute_loss(self, outputs, labels):
        """Reference-API loss on GPT.forward's outputs (trainer.py:139-167)."""
        if not isinstance(outputs, (list, tuple)) or len(outputs) == 1:
            return F.cross_entropy(outputs.float().reshape(-1, outputs.size(-1)), labels.reshape(-1),
                                   ignore_index=self.pad_id)
        logits, halt, qs, targets = outputs
        token = F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), labels.reshape(-1),
                                ignore_index=self.pad_id)
        q_cont = torch.zeros((), device=logits.device)
        if len(qs) > 0:
            for i in range(len(qs)):
                q_cont = q_cont + F.binary_cross_entropy_with_logits(qs[i][..., 1], targets[i])
            q_cont = q_cont / len(qs)
        avg_halt = halt / len(qs) if len(qs) > 0 else 0
        total = token + q_cont + avg_halt
        return total, token.item(), (q_cont + avg_halt).item()

    def train_step(self, micro_batches):
        """One optimizer step over `micro_batches` (list of (input_ids, labels) with 1 extra token).

        Returns device tensors (total, token, q) summed over micro-batches."""
        self.model.train()
        acc = torch.zeros(3, device=self.device)
        inv = 1.0 / len(micro_batches)
        for src, tgt in micro_batches:
            src = src.to(self.device, non_blocking=True)
            tgt = tgt.to(self.device, non_blocking=True)
            total, tok, q = self.model.forward_loss(src[:, :-1], tgt[:, 1:].contiguous())
            (total * inv).backward()
            acc += torch.stack([total.detach() * inv, tok.detach() * inv, q.detach()])
        if self.log_grad_norm and self.is_main_process:
            norms = [p.grad.norm() for p in self.model.parameters() if p.grad is not None]
            print(f"Gradient norm: {torch.stack(norms).norm().item():.4f}")
        if self.grad_clip is not None:
            torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.grad_clip)
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        if self.scheduler is not None:
            self.scheduler.step()
        self.global_step += 1
        return acc

    def train(self):
        val_every = self.cfg.training.get("val_every_n_steps", 1000) if hasattr(self.cfg.training, "get") else 1000
        it = iter(self.train_loader)
        while self.global_step < self.total_steps:
            micro = []
            for _ in range(self.grad_accum_steps):
                try:
                    batch = next(it)
                except StopIteration:
                    it = iter(self.train_loader)
                    batch = next(it)
                micro.append((batch["src"], batch["tgt"]))
            acc = self.train_step(micro)
            if self.is_main_process:
                tot, tok, q = acc.tolist()
                lr = self.optimizer.param_groups[0]["lr"]
                self.logger.log({"Loss/train_total": tot, "Loss/train_token": tok, "Loss/train_q": q, "lr": lr},
                                self.global_step)
            final = self.global_step == self.total_steps
            if (self.global_step > 0 and self.global_step % val_every == 0) or final:
                val = self._validate_loss(self.val_loader)  # averaged over ranks: every rank decides alike
                self.logger.log({"Loss/val_fineweb": val}, self.global_step)
                if val < self.best_metric:
                    self.best_metric, self.best_epoch = val, self.global_step
                    self.save_checkpoint(self.best_model_path, self.global_step)  # every rank: may gather
                    self.epochs_no_improve = 0
                else:
                    self.epochs_no_improve += 1
                if self.is_ddp:
                    import torch.distributed as dist

                    dist.barrier()
                if 0 < self.early_stopping_patience <= self.epochs_no_improve:
                    break
        if self.is_main_process:
            print(f"Training complete. Best Loss: {self.best_metric:.4f}")

    def _inputs_labels(self, batch):
        """(inputs, next-token labels) on the device from a batch of either collate schema."""
        if "src" in batch:
            src, tgt = batch["src"], batch["tgt"]
        elif "input_ids" in batch:
            src, tgt = batch["input_ids"], batch["labels"]
        else:
            raise KeyError("a batch needs 'src'/'tgt' (token stream) or 'input_ids'/'labels' (multiple choice)")
        src = src.to(self.device, non_blocking=True)
        tgt = tgt.to(self.device, non_blocking=True)
        return src[:, :-1], tgt[:, 1:].contiguous()

    @torch.no_grad()
    def _evaluate(self, dataloader):
        """Mean token loss over the loader's batches (trainer.py:272-292) and, for multiple-choice batches,
        (correct by summed loss, correct by mean loss, items). Data-parallel ranks are averaged / summed."""
        self.model.eval()
        total = torch.zeros((), device=self.device)
        mc = torch.zeros(3, device=self.device, dtype=torch.float64)
        count = 0
        for batch in dataloader:
            inp, lab = self._inputs_labels(batch)
            _, tok, _ = self.model.forward_loss(inp, lab)
            total += tok
            count += 1
            if "example_indices" in batch:
                mc += self._score_choices(inp, lab, batch["example_indices"], batch["correct_labels"])
        avg = total / count if count > 0 else total
        if self.is_ddp:
            import torch.distributed as dist

            dist.all_reduce(avg, op=dist.ReduceOp.AVG)
            dist.all_reduce(mc, op=dist.ReduceOp.SUM)
        self.model.train()
        return avg.item(), mc.tolist()

    def _score_choices(self, inp, lab, owner, correct):
        """Per item, the ending with the lowest summed / mean loss over its scored tokens."""
        losses = self.model.token_losses(inp, lab)
        scored = (lab != self.pad_id).float()
        tot = losses.sum(dim=1)
        mean = tot / scored.sum(dim=1).clamp_min(1.0)
        owner = owner.to(self.device)
        n_items = int(correct.numel())
        correct = correct.to(self.device)
        res = torch.zeros(3, device=self.device, dtype=torch.float64)
        for i in range(n_items):
            rows = (owner == i).nonzero().flatten()
            if rows.numel() == 0:
                continue
            res[0] += float(torch.argmin(tot[rows]) == correct[i])
            res[1] += float(torch.argmin(mean[rows]) == correct[i])
            res[2] += 1
        return res

    def _validate_loss(self, dataloader):
        loss, _ = self._evaluate(dataloader)
        return loss

    def test(self):
        """Test loss (trainer.py:294-305); multiple-choice loaders also report accuracy."""
        if self.is_main_process:
            print("Testing the model...")
        loss, (acc, acc_norm, n) = self._evaluate(self.test_loader)
        metrics = {"Loss/test": loss}
        if n > 0:
            metrics.update({"Acc/test": acc / n, "Acc/test_norm": acc_norm / n})
        self.test_metrics = metrics
        if self.is_main_process:
            self.logger.log(metrics, self.global_step)
            print(f"Test Loss: {loss:.4f}" + (f"  accuracy {acc / n:.4f} (length-normalised {acc_norm / n:.4f})"
                                              if n > 0 else ""))
        if self.is_ddp:
            import torch.distributed as dist

            dist.barrier()
        return loss

    # ------------------------------------------------------------------ checkpoints
    def _get_model_for_saving(self):
        m = self.model.module if hasattr(self.model, "module") else self.model
        return m._orig_mod if hasattr(m, "_orig_mod") else m

    def save_checkpoint(self, path, epoch):
        """Same dictionary as the reference (trainer.py:311-322), written by rank 0. Call it on every rank:
        a sharded data-parallel optimizer first gathers its state (a collective)."""
        consolidate = getattr(self.optimizer, "consolidate_state_dict", None)
        opt_state = consolidate() if (self.is_ddp and consolidate is not None) else None
        if not self.is_main_process:
            return
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        ck = {"model_state_dict": self._get_model_for_saving().state_dict(),
              "optimizer_state_dict": opt_state if opt_state is not None else self.optimizer.state_dict(),
              "best_metric": self.best_metric, "global_step": self.global_step}
        if self.scheduler is not None:
            ck["scheduler_state_dict"] = self.scheduler.state_dict()
        torch.save(ck, path)

    def load_checkpoint(self, path):
        """Resume from a save_checkpoint() file (model, optimizer state, counters)."""
        ck = torch.load(path, map_location=self.device, weights_only=False)
        self._get_model_for_saving().load_state_dict(ck["model_state_dict"])
        self.optimizer.load_state_dict(ck["optimizer_state_dict"])
        self.best_metric = ck.get("best_metric", float("inf"))
        self.global_step = ck.get("global_step", 0)
        if self.scheduler is not None:
            if "scheduler_state_dict" in ck:
                self.scheduler.load_state_dict(ck["scheduler_state_dict"])
            else:  # a checkpoint of the reference's format: replay the schedule up to the saved step
                for _ in range(self.global_step):
                    self.scheduler.step()
        return ck
