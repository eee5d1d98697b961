#!/usr/bin/env python
"""Training-throughput benchmark of the rGPT step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gpt-small|rgpt-small|gpt-350m]
                    [--impl ours|reference]

One "step" is one optimizer step of the named workload on every rank: forward,
cross entropy (+ rGPT halting losses), backward and the Muon/AdamW update, all
on the native sm_100a kernels. The default workload is the gpt-small training
step (d_model 512, 8 heads, 8 layers, squared-ReLU FFN, RMSNorm pre-norm,
f_rmsnorm QK norm, RoPE, G1 gate, vocab 50304, seq 1024, micro-batch 16,
Muon for 2-D weights + AdamW) on synthetic uniform token ids with
random-init weights, dropout 0.1 (the reference's model configs). Multi-GPU runs
(torchrun) are weak-scaling data parallel: 16 sequences per GPU, gradients
averaged over NCCL by DistMuon. The step is replayed as one CUDA graph on one
GPU and on every rank of a multi-GPU run (rgpt_b200.graph.GraphedTrainStep; the
graph holds the collectives); --eager issues every kernel from Python instead.

Printed (rank 0, one JSON line): value = whole-job tokens/s with inputs resident
in HBM; e2e = tokens/s through the public API with the token ids copied from
pinned host memory and the loss read back every step; roofline = achieved
TF/s of the tcgen05 GEMM kernel (every launch of K eager steps issued on one
stream, CUDA events around each) vs the measured bf16 peak; cpu_baseline = the CPU oracle (a restatement
of the reference's PyTorch step) timed on this host's cores on a bounded sample.

--impl reference times that CPU implementation of the same workload on all host
cores (rank 0 only; one 1024-token sequence per step) and prints the same line
with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# dropout 0.1: the value of every model config of the reference (conf/model/*.yaml)
COMMON = dict(detach_recur=False, max_seq_len=1024, dropout=0.1, norm_type="rmsnorm", norm_eps=1e-5,
              qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, pad_token_id=-100,
              tie_word_embeddings=False, vocab_size=50304)
WORKLOADS = {
    "gpt-small": dict(cfg=dict(COMMON, name="gpt", n_layers=8, n_recur=1, cal_halt_loss=False, n_heads=8,
                               d_model=512, use_layer_scale=False), B=16, T=1024, accum=1),
    "rgpt-small": dict(cfg=dict(COMMON, name="rgpt", n_layers=2, n_recur=4, cal_halt_loss=True, n_heads=8,
                                d_model=512, use_layer_scale=True), B=16, T=1024, accum=4),
    "gpt-350m": dict(cfg=dict(COMMON, name="gpt", n_layers=24, n_recur=1, cal_halt_loss=False, n_heads=16,
                              d_model=1024, use_layer_scale=False), B=16, T=1024, accum=1),
}
OPT = dict(lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)  # conf/training/default.yaml
# Measured DRAM traffic (read + write) per tcgen05 GEMM launch, averaged over the 168 GEMM
# launches of one gpt-small step: ncu dram__bytes_read.sum + dram__bytes_write.sum
# (profiles/gemm_gpt_small_step_dram.md). Workloads without a capture report null.
GEMM_TRAFFIC = {"gpt-small": 84.33e6}


def flops_per_token(cfg, T):
    """Algorithmic training FLOPs per token (fwd + bwd = 3x fwd), causal attention counted at half."""
    d, L, R, V = cfg["d_model"], cfg["n_layers"], cfg.get("n_recur", 1), cfg["vocab_size"]
    H = cfg["n_heads"]
    per_layer = 2 * d * d * 4 + 2 * d * 4 * d * 2 + 2 * 64 * 64 * H + 2 * 2 * T * d / 2
    fwd = L * R * per_layer + 2 * d * V
    if cfg.get("cal_halt_loss") and R > 1:
        fwd += R * 2 * d * V  # per-recurrence lm_head forwards (their CE is discarded but computed)
        return 3 * (fwd - R * 2 * d * V) + R * 2 * d * V
    return 3 * fwd


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"rgpt_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception as e:  # nvidia-smi missing: report no clocks rather than fail the bench
            log("clock sampling unavailable:", e)
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                     parts[4:8]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------ ours
def run_ours(args, wl):
    from rgpt_b200 import _lib
    from rgpt_b200 import native as nv
    from rgpt_b200.model import GPT
    from rgpt_b200.optimizer import DistMuon, Muon, trainer_param_groups

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the native path has no CPU fallback)")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg, B, T, accum = dict(wl["cfg"]), wl["B"], wl["T"], wl["accum"]
    if args.dropout is not None:
        cfg["dropout"] = args.dropout
    torch.manual_seed(1234)
    model = GPT(**cfg).to(dev).train()
    opt = (DistMuon if world > 1 else Muon)(trainer_param_groups(model), **OPT)
    g = torch.Generator().manual_seed(1000 + rank)
    n_batches = 4
    host = [torch.randint(0, cfg["vocab_size"], (accum, B, T + 1), generator=g).pin_memory() for _ in range(n_batches)]
    dev_batches = [h.to(dev) for h in host]
    ids_dev = torch.empty_like(dev_batches[0])
    inv_accum = 1.0 / accum

    graphed = None
    if not args.eager:
        # the whole step as one CUDA graph; 2 eager warm-up steps build the optimizer state first
        from rgpt_b200.graph import GraphedTrainStep

        graphed = GraphedTrainStep(model, opt, B, T, accum, warmup=2)
        step, step_eager = graphed, graphed.eager
    else:
        def step(ids):
            opt.zero_grad(set_to_none=True)
            total = None
            for a in range(accum):
                total, _, _ = model.forward_loss(ids[a, :, :-1], ids[a, :, 1:])
                (total * inv_accum).backward()
            opt.step()
            return total
        step_eager = step

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for i in range(args.warmup):
        step(dev_batches[i % n_batches])
    barrier()

    # ---- device-resident timing
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.4)
    _lib.launch_count = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for i in range(args.steps):
        last = step(dev_batches[i % n_batches])
    e1.record()
    barrier()
    launches = _lib.launch_count // args.steps
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    clocks = sampler.stop() if sampler else None
    loss_val = last.item()
    if not math.isfinite(loss_val):
        raise SystemExit(f"non-finite loss {loss_val}")

    # ---- end-to-end through the public API: pinned host ids -> device, loss read back every step
    loss_host = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    barrier()
    e0.record()
    for i in range(args.steps):
        if graphed is not None:
            total = step(host[i % n_batches])  # H2D copy into the graph's static id buffer
        else:
            ids_dev.copy_(host[i % n_batches], non_blocking=True)
            total = step(ids_dev)
        loss_host[i:i + 1].copy_(total.detach().reshape(1), non_blocking=True)
    e1.record()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    # ---- GEMM kernel roofline: CUDA events around every tcgen05 GEMM launch of K steps, issued launch by
    # launch so each GEMM gets its own events, and on one stream (no side-stream mask or optimizer work
    # running beside a GEMM and stretching its measured duration); the timed steps above keep the overlap
    eng = model.engine()
    eng.overlap_masks, opt.concurrent = False, False
    nv.gemm_events = []
    barrier()
    for i in range(args.steps):
        step_eager(dev_batches[i % n_batches])
    barrier()
    ev, nv.gemm_events = nv.gemm_events, None
    eng.overlap_masks, opt.concurrent = True, True
    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in ev)
    gemm_flops = sum(f for _, _, f in ev)
    from rgpt_b200.peaks import load_peaks

    peaks = load_peaks()
    gemm_tfs = gemm_flops / (gemm_ms * 1e-3) / 1e12
    tokens = B * T * accum
    value = world * tokens / (ms * 1e-3)
    e2e = world * tokens / (ms_e2e * 1e-3)
    fpt = flops_per_token(cfg, T)
    res = {
        "metric": "train tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: uniform random token ids in [0, 50304), random-init weights (seeded)",
        "config": {"workload": args.workload, "model": cfg["name"], "d_model": cfg["d_model"],
                   "n_layers": cfg["n_layers"], "n_recur": cfg.get("n_recur", 1), "n_heads": cfg["n_heads"],
                   "vocab": cfg["vocab_size"], "seq_len": T, "micro_batch": B, "grad_accum": accum,
                   "global_batch": B * accum * world, "parallelism": f"dp{world}",
                   "optimizer": "Muon (5 NS steps) + AdamW", "dropout": cfg["dropout"],
                   "launch": "one CUDA graph replay per step" if graphed is not None else "eager",
                   "l2": "no flush: each step's working set (activations + weights) is several GB, far above "
                         "the 126 MB L2"},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": host[0].numel() * 8,
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "model_tflops": round(fpt * value / world / 1e12, 1),
        "loss_last_step": round(loss_val, 4),
        "roofline": {"kernel": "gemm_bf16_tc_kernel (all launches)", "bound": "tensor",
                     "method": "CUDA events around each GEMM launch of eager steps issued on one stream",
                     "achieved": round(gemm_tfs, 1), "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": round(gemm_tfs / peaks["bf16_tflops_sustained"], 3),
                     "peak_source": peaks["source"] + " (sustained bf16: kernels timed inside a long step)",
                     "launches_per_step": len(ev) // args.steps,
                     "gemm_share_of_step": round(gemm_ms / args.steps / ms, 3),
                     "traffic": GEMM_TRAFFIC.get(args.workload),
                     "traffic_unit": "bytes per launch: DRAM read + write of all GEMM launches of one step / "
                                     "launches, from one ncu capture (profiles/gemm_gpt_small_step_dram.md)"},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg, T, budget_s=args.cpu_budget)
    if dist is not None:
        dist.barrier(device_ids=[local])
        if graphed is not None:
            graphed.release()  # a graph holding NCCL collectives must go before its process group
            torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------------------ CPU reference
def _cpu_train_steps(cfg, T, n_steps, threads):
    """Time the oracle (CPU restatement of the reference's PyTorch step) on one 1024-token sequence."""
    from oracle import ref_ops as O
    from rgpt_b200.model import GPT

    torch.set_num_threads(threads)
    torch.manual_seed(1234)
    m = GPT(**cfg)
    params = {k: v for k, v in m.state_dict().items() if v.is_floating_point() and not k.endswith((".eps", "inv_freq"))}
    del m
    g = torch.Generator().manual_seed(7)
    batches = [[(ids, ids)] for ids in torch.randint(0, cfg["vocab_size"], (n_steps, 1, T + 1), generator=g)]
    times = []
    params = {k: v.clone().requires_grad_(True) for k, v in params.items()}
    opt = O.OracleMuon(params, **OPT)
    for micro in batches:
        t0 = time.perf_counter()
        ids, labels = micro[0]
        out = O.gpt_forward(params, ids[:, :-1], cfg, labels=labels[:, 1:].contiguous(), training=True,
                            drop_seed="torch")
        loss, _ = O.compute_loss(out, labels[:, 1:])
        grads = dict(zip(params, torch.autograd.grad(loss, list(params.values()), allow_unused=True)))
        opt.step({k: v for k, v in grads.items() if v is not None})
        times.append(time.perf_counter() - t0)
    return times


def cpu_baseline(cfg, T, budget_s=30.0):
    threads = os.cpu_count() or 1
    times = _cpu_train_steps(cfg, T, 1, threads)  # warm-up step, also sizes the sample
    n = max(1, min(5, int(budget_s / max(times[0], 1e-3))))
    times = _cpu_train_steps(cfg, T, n, threads)
    per_step = statistics.median(times)
    return {"value": round(T / per_step, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} oracle training steps (forward, CE, backward, Muon+AdamW, dropout "
                      f"{cfg['dropout']} from torch's generator) on 1 sequence x {T} tokens, "
                      f"fp32 CPU, median step {per_step:.2f} s"}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, T = dict(wl["cfg"]), wl["T"]
    if args.dropout is not None:
        cfg["dropout"] = args.dropout
    threads = os.cpu_count() or 1
    _cpu_train_steps(cfg, T, max(1, min(args.warmup, 2)), threads)
    times = _cpu_train_steps(cfg, T, args.steps, threads)
    ms = 1000.0 * statistics.mean(times)
    value = T / (ms * 1e-3)
    res = {
        "impl": "reference", "metric": "train tokens/s", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: uniform random token ids, random-init weights (seeded)",
        "config": {"workload": args.workload, "model": cfg["name"], "seq_len": T, "micro_batch": 1,
                   "parallelism": "cpu", "dropout": cfg["dropout"],
                   "note": "one 1024-token sequence per step (bounded CPU sample)"},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} oracle training steps on 1 x {T} tokens (fp32, all host threads)"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="gpt-small")
    ap.add_argument("--cpu-budget", type=float, default=30.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="issue every kernel from Python (no CUDA graph)")
    ap.add_argument("--dropout", type=float, default=None,
                    help="dropout rate of the embedding, attention probabilities and residual branches "
                         "(default: the workload's)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        log("note: warm-up raised to 3 steps")
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
