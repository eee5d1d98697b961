#!/usr/bin/env python
"""Benchmarks of the rGPT training step on B200; each run prints one JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Workloads (sizes in rgpt_b200/workloads.py):
  gpt-small (default), rgpt-small, gpt-350m
      One optimizer step of the training step on every rank: forward, cross entropy (+ rGPT halting
      losses), backward and the Muon/AdamW update, all on the native sm_100a kernels, replayed as one
      CUDA graph (--eager issues every kernel from Python). Synthetic uniform token ids, random-init
      weights, dropout 0.1 (the reference's model configs). Under torchrun: weak-scaling data parallel,
      16 sequences per GPU, gradients averaged over NCCL by DistMuon.
      value = whole-job tokens/s with the ids resident in HBM; e2e = the same through the public API
      with the ids copied from pinned host memory and the loss read back every step; roofline = the
      weight-gradient GEMMs (the CTA-pair split-K reduce-add instantiation of gemm_bf16_tc_kernel, the
      largest share of the step) timed launch by launch with CUDA events inside eager steps;
      gemm_classes = the same for every GEMM shape of the step; optimizer = the Muon + AdamW step alone.
  muon-step
      The single-matrix Muon step: W [2048, 512], 5 Newton-Schulz steps, plus AdamW on a 512-vector
      (milliseconds per step, CUDA-graph replays and eager); roofline = the Newton-Schulz GEMMs.
  ffn-sweep
      FusedLinearActivationFunction forward + backward over M in {8192 .. 65536} x four activations
      (aggregate TFLOP/s); roofline = the fc1 GEMM with the activation epilogue at the largest M.
  kernels
      One launch of each hot kernel of the gpt-small step (GEMM classes, attention, row kernels,
      optimizer), each timed alone with CUDA events after an L2 flush, with its achieved TFLOP/s or GB/s
      against the measured peaks. --only NAME runs one case and --launches N its launch count, for a
      profiler capture of exactly that kernel.

--impl reference times the CPU implementation of the same workload (the oracle: a restatement of the
reference's PyTorch step) on all host cores, rank 0 only, and prints the same line with "impl":
"reference". cpu_baseline in our line is the same measurement on a bounded sample.
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
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from rgpt_b200.workloads import FFN_SWEEP, MUON_SINGLE, OPT, WORKLOADS  # noqa: E402

TRAIN_WORKLOADS = list(WORKLOADS)
ALL_WORKLOADS = TRAIN_WORKLOADS + ["muon-step", "ffn-sweep", "kernels"]

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per weight-gradient GEMM launch, averaged
# over one gpt-small step's 33 launches (8 each of the fc1, fc2, out_proj and QKV shapes, 1 lm_head), from
# one ncu capture of each shape (bench.py --workload kernels --only wgrad_*); absent for other workloads.
WGRAD_TRAFFIC_PER_LAUNCH = {"gpt-small": 145.2e6}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    from rgpt_b200.peaks import load_peaks as lp

    return lp()


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event reasons of this process's GPU, sampled every 10 ms through NVML
    on a background thread while the timed region runs (nvidia-smi's 200 ms loop when NVML is
    unavailable)."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, device_index: int = 0, period_s: float = 0.01):
        self.device_index, self.period = device_index, period_s
        self.samples, self.reasons = [], set()
        self.power = []
        self.mx = None
        self._stop = threading.Event()
        self._thread = None
        self._smi = None
        self.source = None

    def _handle(self):
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device_index)
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            try:
                return pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
            except Exception:
                try:
                    return pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(uuid))
                except Exception:
                    pass
        return pynvml.nvmlDeviceGetHandleByIndex(self.device_index)

    def start(self):
        try:
            import pynvml

            h = self._handle()
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        r = int(get_reasons(h))
                        for name, bit in self.REASONS:
                            if r & bit:
                                self.reasons.add(name)
                        self.power.append(pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0)
                    except Exception:
                        pass
                    self._stop.wait(self.period)

            self.source = "nvml, every 10 ms"
            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception as e:
            log("NVML clock sampling unavailable, using nvidia-smi:", e)
            self._start_smi()

    def _start_smi(self):
        fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")
        try:
            self._path = os.path.join(tempfile.gettempdir(), f"rgpt_clocks_{os.getpid()}.csv")
            self._fh = open(self._path, "w")
            self._smi = subprocess.Popen(["nvidia-smi", "-i", str(self.device_index), f"--query-gpu={fields}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self._fh,
                                         stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi, every 200 ms"
        except Exception as e:
            log("clock sampling unavailable:", e)

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        elif self._smi is not None:
            self._smi.terminate()
            try:
                self._smi.wait(timeout=5)
            except Exception:
                self._smi.kill()
            self._fh.close()
            with open(self._path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 7:
                        continue
                    try:
                        self.samples.append(float(parts[0]))
                        self.mx = float(parts[1])
                        self.power.append(float(parts[2]))
                    except ValueError:
                        continue
                    for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                          "sw_power_cap"), parts[3:7]):
                        if val.lower().startswith("active"):
                            self.reasons.add(name)
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.mx, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "power_w_max": round(max(self.power), 1) if self.power else None,
                "source": self.source}


# ------------------------------------------------------------------------------------------ helpers
def flops_per_token(cfg, T):
    """Algorithmic training FLOPs per token (fwd + bwd = 3x fwd), causal attention counted at half; rGPT's
    per-recurrence lm_head forwards (their logits feed only the halting targets) counted once."""
    d, L, R, V = cfg["d_model"], cfg["n_layers"], cfg.get("n_recur", 1), cfg["vocab_size"]
    H = cfg["n_heads"]
    per_layer = 2 * d * d * 4 + 2 * d * 4 * d * 2 + 2 * 64 * 64 * H + 2 * 2 * T * d / 2
    fwd = L * R * per_layer + 2 * d * V
    if cfg.get("cal_halt_loss") and R > 1:
        return 3 * fwd + R * 2 * d * V
    return 3 * fwd


EPI_NAMES = {0: "store_bf16", 1: "store_f32", 2: "accum_f32 (split-K reduce-add)", 3: "act_fwd", 4: "act_bwd",
             5: "resid_f32", 6: "poly_bf16", 7: "bias_sigmoid", 8: "poly_f32", 9: "argmax"}


def is_wgrad(key):
    """The weight-gradient GEMMs: fp32 reduce-add into the gradient arena, both operands read MN-major,
    256 x 256 CTA-pair tiles (wide M and N, K >= 2048 tokens), split K."""
    epi, M, N, K, batch = key
    return epi == 2 and batch == 1 and M > 128 and N > 128 and K >= 2048


def gemm_bytes(key):
    """Algorithmic DRAM bytes of one GEMM launch: each operand read once, the output written once (read
    too when the epilogue adds to it)."""
    epi, M, N, K, batch = key
    out = {0: 2, 1: 4, 2: 8, 3: 4, 4: 4, 5: 12, 6: 4, 7: 2, 8: 8, 9: 0}[epi]
    extra_c = {4: 2, 6: 2, 8: 4}.get(epi, 0)
    return batch * (2 * M * K + 2 * N * K + (out + extra_c) * M * N)


class L2Flush:
    """Writes a 256 MB buffer (twice the 126 MB L2), then reads another 256 MB one, so the next timed
    kernel starts from DRAM with an L2 of clean lines. Without the read pass L2 would still hold ~126 MB
    of the write's dirty lines, and their write-back would be charged to the timed kernel."""

    def __init__(self, dev):
        self.buf = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
        self.rd = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
        self.out = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)
        torch.sum(self.rd, dim=0, out=self.out)


def time_launches(fn, n, flush=None):
    """Median CUDA-event time (ms) of n calls of fn on the current stream, each after an L2 flush."""
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(n):
        if flush is not None:
            flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def graph_time(fn, reps=10):
    """ms per call of fn, from CUDA-graph replays of `reps` back-to-back calls (launch gaps removed)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _cuda_device():
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the native path has no CPU fallback)")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    return torch.device("cuda", local), local


# ------------------------------------------------------------------------------------------ training step
def run_train(args, wl):
    from rgpt_b200 import _lib
    from rgpt_b200 import native as nv
    from rgpt_b200.model import GPT
    from rgpt_b200.optimizer import DistMuon, Muon, trainer_param_groups

    dev, local = _cuda_device()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
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
    opt = (DistMuon(trainer_param_groups(model), sharded_state=args.dp == "sharded", **OPT) if world > 1
           else Muon(trainer_param_groups(model), **OPT))
    g = torch.Generator().manual_seed(1000 + rank)
    n_batches = 4
    host = [torch.randint(0, cfg["vocab_size"], (accum, B, T + 1), generator=g).pin_memory() for _ in range(n_batches)]
    dev_batches = [h.to(dev) for h in host]
    ids_dev = torch.empty_like(dev_batches[0])
    inv_accum = 1.0 / accum

    graphed = None
    if not args.eager:
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
    if args.profile_region:
        # K eager steps inside cudaProfilerStart/Stop, for a profiler run with --profile-from-start off
        torch.cuda.cudart().cudaProfilerStart()
        for i in range(args.steps):
            step_eager(dev_batches[i % n_batches])
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        if dist is not None:
            if graphed is not None:
                graphed.release()
            dist.destroy_process_group()
        return

    # ---- device-resident timing: exactly K steps between barriers, clocks sampled meanwhile
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    _lib.launch_count = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for i in range(args.steps):
        last = step(dev_batches[i % n_batches])
    e1.record()
    barrier()
    clocks = sampler.stop() if sampler else None
    launches = _lib.launch_count // args.steps
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    loss_val = last.item()
    if not math.isfinite(loss_val):
        raise SystemExit(f"non-finite loss {loss_val}")

    # ---- end to end through the public API: pinned host ids -> device, loss read back every step
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

    # ---- GEMM classes: CUDA events around every GEMM launch of eager steps issued on one stream (no
    # side-stream mask or optimizer work runs beside a GEMM inside its events); the timed steps above
    # keep the overlap
    eng = model.engine()
    eng.overlap_masks, opt.concurrent = False, False
    n_ev_steps = max(1, min(args.steps, 5))
    nv.gemm_events = []
    barrier()
    for i in range(n_ev_steps):
        step_eager(dev_batches[i % n_batches])
    barrier()
    ev, nv.gemm_events = nv.gemm_events, None
    classes = {}
    for a, b, f, key in ev:
        c = classes.setdefault(key, [0.0, 0.0, 0])
        c[0] += a.elapsed_time(b)
        c[1] += f
        c[2] += 1
    # ---- the optimizer step alone (Muon + AdamW on the step's gradients), eager, one stream
    opt_ms = time_launches(opt.step, 5) if world == 1 else None
    eng.overlap_masks, opt.concurrent = True, True

    peaks = load_peaks()
    sustained, burst = peaks["bf16_tflops_sustained"], peaks["bf16_tflops"]
    wg = [(k, v) for k, v in classes.items() if is_wgrad(k)]
    wg_ms = sum(v[0] for _, v in wg)
    wg_flops = sum(v[1] for _, v in wg)
    wg_n = sum(v[2] for _, v in wg)
    wg_tfs = wg_flops / (wg_ms * 1e-3) / 1e12 if wg_ms > 0 else 0.0
    wg_bytes = sum(gemm_bytes(k) * v[2] for k, v in wg) / max(wg_n, 1)
    all_ms = sum(v[0] for v in classes.values())
    top = sorted(classes.items(), key=lambda kv: -kv[1][0])[:8]
    gemm_classes = [{"M": k[1], "N": k[2], "K": k[3], "batch": k[4], "epilogue": EPI_NAMES[k[0]],
                     "launches_per_step": v[2] // n_ev_steps, "us_per_launch": round(1e3 * v[0] / v[2], 1),
                     "tflops": round(v[1] / (v[0] * 1e-3) / 1e12, 1),
                     "frac_of_sustained": round(v[1] / (v[0] * 1e-3) / 1e12 / sustained, 3)} for k, v in top]

    tokens = B * T * accum
    value = world * tokens / (ms * 1e-3)
    e2e = world * tokens / (ms_e2e * 1e-3)
    fpt = flops_per_token(cfg, T)
    traffic = WGRAD_TRAFFIC_PER_LAUNCH.get(args.workload)
    res = {
        "metric": "train tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: uniform random token ids in [0, 50304), random-init weights (seeded)",
        "config": {"workload": args.workload, "model": cfg["name"], "d_model": cfg["d_model"],
                   "n_layers": cfg["n_layers"], "n_recur": cfg.get("n_recur", 1), "n_heads": cfg["n_heads"],
                   "vocab": cfg["vocab_size"], "seq_len": T, "micro_batch": B, "grad_accum": accum,
                   "global_batch": B * accum * world, "parallelism": f"dp{world}",
                   "dp_step": (args.dp if world > 1 else None),
                   "optimizer": "Muon (5 NS steps) + AdamW", "dropout": cfg["dropout"],
                   "launch": "one CUDA graph replay per step" if graphed is not None else "eager",
                   "l2": "no flush: each step's working set (activations + weights) is several GB, far above "
                         "the 126 MB L2"},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": host[0].numel() * 8,
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "model_tflops": round(fpt * value / world / 1e12, 1),
        "loss_last_step": round(loss_val, 4),
        "roofline": {"kernel": "gemm_bf16_tc_kernel<256,6,MN,MN,ACCUM_F32,pair>: the weight-gradient GEMMs "
                               "(CTA-pair 256x256 tiles, split K, TMA bulk reduce-add into the fp32 gradients)",
                     "bound": "tensor", "method": f"CUDA events around each launch of {n_ev_steps} eager steps "
                                                  "issued on one stream",
                     "launches_per_step": wg_n // n_ev_steps,
                     "achieved": round(wg_tfs, 1), "peak": sustained, "unit": "TFLOP/s",
                     "frac": round(wg_tfs / sustained, 3), "frac_of_burst": round(wg_tfs / burst, 3),
                     "peak_source": peaks["source"] + " (sustained bf16 for kernels timed inside a step; "
                                                      "burst beside it)",
                     "share_of_step": round(wg_ms / n_ev_steps / ms, 3),
                     "algorithmic_bytes_per_launch": round(wg_bytes),
                     "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu)"},
        "gemm_classes": gemm_classes,
        "gemm_share_of_step": round(all_ms / n_ev_steps / ms, 3),
        "optimizer": {"ms": round(opt_ms, 4) if opt_ms is not None else None,
                      "what": "Muon (momentum, 5 batched Newton-Schulz steps per shape class, apply) + AdamW "
                              "over every parameter, eager, one stream"},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_train_baseline(cfg, T, budget_s=args.cpu_budget)
    if dist is not None:
        dist.barrier(device_ids=[local])
        if graphed is not None:
            graphed.release()  # a graph holding NCCL collectives must go before its process group
            torch.cuda.synchronize()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------------------ Muon step
def _muon_inputs():
    c = MUON_SINGLE
    g = torch.Generator().manual_seed(c["seed"])
    R, C = c["shape"]
    W = torch.randn(R, C, generator=g) * c["w_std"]
    G = torch.randn(R, C, generator=g) * c["g_std"]
    p = c["adam_p_mean"] + torch.randn(c["adam_n"], generator=g) * c["adam_p_std"]
    gp = torch.randn(c["adam_n"], generator=g) * c["adam_g_std"]
    return W, G, p, gp


def run_muon_step(args):
    from rgpt_b200 import native as nv
    from rgpt_b200.optimizer import Muon

    dev, _ = _cuda_device()
    c = MUON_SINGLE
    W0, G0, p0, gp0 = _muon_inputs()
    W = torch.nn.Parameter(W0.to(dev))
    P = torch.nn.Parameter(p0.to(dev))
    W.grad, P.grad = G0.to(dev), gp0.to(dev)
    # the reference call: muon_update (momentum 0.95, Nesterov, 5 NS steps) then p.add_(update, alpha=-lr),
    # plus foreach_adamw_step on the vector; no weight decay, Muon lr = lr
    opt = Muon([{"params": [W], "use_muon": True}, {"params": [P], "use_muon": False, "weight_decay": 0.0}],
               lr=c["lr"], weight_decay=0.0, momentum=c["momentum"], muon_lr_multiplier=1.0, ns_steps=c["ns_steps"])
    opt.use_device_hparams()

    def one():
        opt.stage_device_hparams()
        opt.step()

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    eager_ms = time_launches(one, max(args.steps, 5))
    # the step captured as a CUDA graph (the per-step scalars staged into the device block before replay)
    opt.stage_device_hparams()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        opt.step()
    for _ in range(3):
        opt.stage_device_hparams()
        g.replay()
    sampler = ClockSampler(dev.index)
    sampler.start()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        opt.stage_device_hparams()
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: the gradient from pinned host memory, the updated weight back to it, every step
    Gh, Wh = G0.clone().pin_memory(), torch.empty_like(W0).pin_memory()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        W.grad.copy_(Gh, non_blocking=True)
        opt.stage_device_hparams()
        g.replay()
        Wh.copy_(W.detach(), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.steps
    # the Newton-Schulz iteration alone (one persistent chain kernel, or the batched GEMMs), on a
    # workspace of this matrix's shape holding a normalised input
    from rgpt_b200.optimizer import NS_IMPL, _NSWorkspace, newton_schulz_batched

    R, C = c["shape"]
    ws = _NSWorkspace(1, min(R, C), max(R, C), dev)
    ws.X[0, :min(R, C), :max(R, C)].copy_((G0 if R <= C else G0.t()).to(dev) / G0.norm())
    ns_ms = time_launches(lambda: newton_schulz_batched(ws, c["ns_steps"]), 20)
    r, cc = min(R, C), max(R, C)
    ns_flops = c["ns_steps"] * (2 * r * r * cc + 2 * r ** 3 + 2 * r * r * cc)
    peaks = load_peaks()
    ns_tfs = ns_flops / (ns_ms * 1e-3) / 1e12
    res = {
        "metric": "NorMuon step ms", "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: W [2048, 512] ~ N(0, 0.02), G ~ N(0, 1) * 1e-2 (seed 0); AdamW 512-vector",
        "config": {"workload": "muon-step", "shape": list(c["shape"]), "ns_steps": c["ns_steps"],
                   "momentum": c["momentum"], "lr": c["lr"], "nesterov": True, "adamw_vector": c["adam_n"],
                   "launch": "one CUDA graph replay per step", "eager_ms": round(eager_ms, 4),
                   "l2": "no flush: the working set (a few MB) stays in L2, as it does inside a training step"},
        "e2e": {"value": round(ms_e2e, 4), "unit": "ms", "h2d_bytes_per_step": G0.numel() * 4,
                "d2h_bytes_per_step": W0.numel() * 4},
        "gpu_launches": 5 if NS_IMPL == "chain" else 19,
        "roofline": {"kernel": ("ns_chain_kernel: the whole Newton-Schulz iteration (A = X X^T; b A + c A^2; a X + B X, "
                                "5 steps) in one persistent launch") if NS_IMPL == "chain" else
                               "gemm_bf16_tc_kernel: the 15 Newton-Schulz GEMMs (A = X X^T; b A + c A^2; a X + B X)",
                     "bound": "tensor", "achieved": round(ns_tfs, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(ns_tfs / peaks["bf16_tflops"], 3),
                     "peak_source": peaks["source"] + " (burst bf16: the GEMMs are timed alone)",
                     "ns_gflop": round(ns_flops / 1e9, 2), "ns_us": round(ns_ms * 1e3, 1), "traffic": None},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_muon_baseline(budget_s=min(args.cpu_budget, 10.0))
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------------------ FFN sweep
def run_ffn_sweep(args):
    from rgpt_b200 import native as nv
    from rgpt_b200.model import FusedLinearActivationFunction

    dev, _ = _cuda_device()
    gen = torch.Generator(device=dev).manual_seed(3)
    K, N = FFN_SWEEP["K"], FFN_SWEEP["N"]
    w1 = (torch.randn(N, K, device=dev, generator=gen) * FFN_SWEEP["w_std"]).bfloat16()
    w2 = (torch.randn(N, K, device=dev, generator=gen) * FFN_SWEEP["w_std"]).bfloat16()  # [N, Out]
    rows, tot_f, tot_ms = [], 0.0, 0.0
    fc1_best = None
    sampler = ClockSampler(dev.index)
    sampler.start()
    for M in FFN_SWEEP["M"]:
        x = torch.randn(M, K, device=dev, generator=gen).bfloat16()
        dy = torch.randn(M, K, device=dev, generator=gen).bfloat16()
        pre = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        post, dpre = torch.empty_like(pre), torch.empty_like(pre)
        out = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
        dw1, dw2 = torch.zeros(N, K, device=dev), torch.zeros(N, K, device=dev)
        dx = torch.empty(M, K, device=dev)
        for name in FFN_SWEEP["activations"]:
            act = nv.act_id(name)

            def fc1():
                nv.gemm(x, w1, pre, epi=nv.EPI_ACT_FWD, act=act, out2=post)

            def fwd_bwd():
                fc1()
                nv.gemm(post, w2.t(), out)
                nv.gemm(post.t(), dy.t(), dw2, epi=nv.EPI_ACCUM_F32, splitk=0)
                nv.gemm(dy, w2, dpre, epi=nv.EPI_ACT_BWD, act=act, c=pre)
                nv.gemm(dpre.t(), x.t(), dw1, epi=nv.EPI_ACCUM_F32, splitk=0)
                nv.gemm(dpre, w1.t(), dx, epi=nv.EPI_STORE_F32)

            t = graph_time(fwd_bwd)
            t1 = graph_time(fc1)
            f = 12.0 * M * K * N
            tot_f += f * args.steps
            tot_ms += t * args.steps
            rows.append({"act": name, "M": M, "us": round(t * 1e3, 1), "tflops": round(f / (t * 1e-3) / 1e12, 1),
                         "fc1_act_fwd_us": round(t1 * 1e3, 1),
                         "fc1_act_fwd_tflops": round(2.0 * M * K * N / (t1 * 1e-3) / 1e12, 1)})
            if M == FFN_SWEEP["M"][-1] and name == "squared_relu":
                fc1_best = 2.0 * M * K * N / (t1 * 1e-3) / 1e12
        del x, dy, pre, post, dpre, out, dx
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    # end to end through the public op on host tensors at the largest M: inputs copied in, dX copied out
    M = FFN_SWEEP["M"][-1]
    xh = torch.randn(M, K).bfloat16().pin_memory()
    dyh = torch.randn(M, K).bfloat16().pin_memory()
    dxh = torch.empty(M, K, dtype=torch.bfloat16).pin_memory()
    w1p, w2p = w1.clone().requires_grad_(True), w2.clone().requires_grad_(True)

    def e2e_once():
        xd = xh.to(dev, non_blocking=True).requires_grad_(True)
        y = FusedLinearActivationFunction.apply(xd, w1p, w2p, "squared_relu")
        y.backward(dyh.to(dev, non_blocking=True))
        dxh.copy_(xd.grad, non_blocking=True)

    e2e_ms = time_launches(e2e_once, max(3, args.steps))
    peaks = load_peaks()
    value = tot_f / (tot_ms * 1e-3) / 1e12
    res = {
        "metric": "fused linear+act fwd+bwd TFLOP/s", "value": round(value, 1), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: X ~ N(0, 1), W1, W2 ~ N(0, 0.02), upstream gradient ~ N(0, 1)",
        "config": {"workload": "ffn-sweep", "M": list(FFN_SWEEP["M"]), "K": K, "N": N,
                   "activations": list(FFN_SWEEP["activations"]),
                   "flops": "12 M K N per forward + backward (fc1 + act, fc2, dW2, dpre, dW1, dX)",
                   "launch": "CUDA-graph replays of 10 passes per case",
                   "l2": "no flush: pre/post/dpre at M >= 16384 are >= 64 MB each, the whole working set above L2"},
        "sweep": rows,
        "e2e": {"value": round(12.0 * M * K * N / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 2 * M * K * 2, "d2h_bytes_per_step": M * K * 2,
                "what": f"FusedLinearActivationFunction.apply + backward on host tensors, M={M}, squared_relu"},
        "gpu_launches": 6 * len(rows),
        "roofline": {"kernel": f"gemm_bf16_tc_kernel<ACT_FWD, squared_relu>: fc1 + activation, M={M}",
                     "bound": "tensor", "achieved": round(fc1_best, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(fc1_best / peaks["bf16_tflops"], 3),
                     "peak_source": peaks["source"] + " (burst bf16)", "traffic": None},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_ffn_baseline(budget_s=min(args.cpu_budget, 15.0))
    print(json.dumps(res), flush=True)


# ------------------------------------------------------------------------------------------ single kernels
def kernel_cases(dev):
    """(name, bound, work per launch (FLOP or algorithmic bytes), setup -> launch fn) of the gpt-small
    step's hot kernels at its sizes: 16 x 1024 tokens, d_model 512, 8 heads, FFN 2048, vocabulary 50304."""
    from rgpt_b200 import native as nv
    from rgpt_b200.optimizer import Muon

    B, T, H, d, F, V = 16, 1024, 8, 512, 2048, 50304
    M = B * T
    g = torch.Generator(device=dev).manual_seed(0)

    def rb(*s):
        return torch.randn(*s, device=dev, generator=g).bfloat16()

    def rf(*s):
        return torch.randn(*s, device=dev, generator=g)

    cases = []

    def add(name, bound, work):
        def deco(setup):
            cases.append((name, bound, work, setup))
            return setup
        return deco

    @add("wgrad_ffn", "tensor", 2.0 * F * d * M)
    def _():
        dpre, hn2, dw = rb(M, F), rb(M, d), torch.zeros(F, d, device=dev)
        return lambda: nv.gemm(dpre.t(), hn2.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)

    @add("wgrad_fc2", "tensor", 2.0 * d * F * M)
    def _():
        dy, post, dw = rb(M, d), rb(M, F), torch.zeros(d, F, device=dev)
        return lambda: nv.gemm(dy.t(), post.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)

    @add("wgrad_out", "tensor", 2.0 * d * d * M)
    def _():
        da, og, dw = rb(M, d), rb(M, d), torch.zeros(d, d, device=dev)
        return lambda: nv.gemm(da.t(), og.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)

    @add("wgrad_qkv", "tensor", 2.0 * 3 * d * d * M)
    def _():
        dqkv, hn, dw = rb(M, 3 * d), rb(M, d), torch.zeros(3 * d, d, device=dev)
        return lambda: nv.gemm(dqkv.t(), hn.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)

    @add("wgrad_lm_head", "tensor", 2.0 * V * d * M)
    def _():
        dl, hf, dw = rb(M, V), rb(M, d), torch.zeros(V, d, device=dev)
        return lambda: nv.gemm(dl.t(), hf.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)

    @add("dx_lm_head", "tensor", 2.0 * M * d * V)
    def _():
        dl, w, dx = rb(M, V), rb(V, d), torch.empty(M, d, device=dev)
        return lambda: nv.gemm(dl, w.t(), dx, epi=nv.EPI_STORE_F32)

    @add("fwd_lm_head", "tensor", 2.0 * M * V * d)
    def _():
        h, w, logits = rb(M, d), rb(V, d), torch.empty(M, V, device=dev, dtype=torch.bfloat16)
        return lambda: nv.gemm(h, w, logits)

    @add("qkv_fwd", "tensor", 2.0 * M * 3 * d * d)
    def _():
        x, w, qkv = rb(M, d), rb(3 * d, d), torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16)
        return lambda: nv.gemm(x, w, qkv)

    @add("fc1_act_fwd", "tensor", 2.0 * M * F * d)
    def _():
        x, w = rb(M, d), rb(F, d)
        pre, post = (torch.empty(M, F, device=dev, dtype=torch.bfloat16) for _ in range(2))
        return lambda: nv.gemm(x, w, pre, epi=nv.EPI_ACT_FWD, act=1, out2=post)

    # the training step's fc1: squared ReLU with the post-activation as its only output
    @add("fc1_sqrelu_post", "tensor", 2.0 * M * F * d)
    def _():
        x, w = rb(M, d), rb(F, d)
        post = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
        return lambda: nv.gemm(x, w, post, epi=nv.EPI_ACT_FWD, act=nv.ACT_SQRELU_POST)

    @add("fc2_resid", "tensor", 2.0 * M * d * F)
    def _():
        post, w, h, x = rb(M, F), rb(d, F), rf(M, d), torch.empty(M, d, device=dev)
        return lambda: nv.gemm(post, w, x, epi=nv.EPI_RESID_F32, c=h)

    @add("attn_fwd", "tensor", 2.0 * 2 * B * H * T * T * 64 / 2)
    def _():
        qk, qkv = rb(M, 2 * d), rb(M, 3 * d)
        gate = torch.sigmoid(rf(M, d)).bfloat16()
        o, og = (torch.empty(M, d, device=dev, dtype=torch.bfloat16) for _ in range(2))
        lse = torch.empty(B, H, T, device=dev)
        return lambda: nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H)

    @add("attn_bwd", "tensor", 5.0 * 2 * B * H * T * T * 64 / 2)
    def _():
        qk, qkv = rb(M, 2 * d), rb(M, 3 * d)
        gate = torch.sigmoid(rf(M, d)).bfloat16()
        o, og = (torch.empty(M, d, device=dev, dtype=torch.bfloat16) for _ in range(2))
        lse = torch.empty(B, H, T, device=dev)
        nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H)
        do, D = rb(M, d), rf(B, H, T)
        dq, dk = torch.zeros(M, d, device=dev), torch.empty(M, d, device=dev)
        dqkv = torch.zeros(M, 3 * d, device=dev, dtype=torch.bfloat16)
        return lambda: nv.attn_bwd(qk, qkv, do, lse, D, dq, dk, dqkv[:, 2 * d:], B, T, H)

    @add("rownorm_fwd", "hbm", M * d * (4 + 2) + d * 4)
    def _():
        x, w, y = rf(M, d), rf(d) * 0.1, torch.empty(M, d, device=dev, dtype=torch.bfloat16)
        return lambda: nv.rownorm_fwd(x, y, nv.NORM_RMS_AFFINE, 1e-5, w=w)

    @add("rownorm_bwd", "hbm", M * d * (4 + 4 + 4 + 4 + 2))
    def _():
        x, w, dy, gi = rf(M, d), rf(d) * 0.1, rf(M, d), rf(M, d)
        go, gb = torch.empty(M, d, device=dev), torch.empty(M, d, device=dev, dtype=torch.bfloat16)
        dw = torch.zeros(d, device=dev)
        return lambda: nv.rownorm_bwd(x, dy, nv.NORM_RMS_AFFINE, 1e-5, go, w=w, g_in=gi, g_bf16=gb, dw=dw)

    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=dev, dtype=torch.float32) / 64))

    # reads the q and k blocks of qkv (v is never touched), writes roped q | k and the normed q
    @add("qkv_prep_fwd", "hbm", M * d * (2 * 2 + 2 * 2 + 2))
    def _():
        qkv = rb(M, 3 * d)
        qk, qn = torch.empty(M, 2 * d, device=dev, dtype=torch.bfloat16), torch.empty(M, d, device=dev,
                                                                                       dtype=torch.bfloat16)
        return lambda: nv.qkv_prep_fwd(qkv, qk, qn, inv_freq, nv.NORM_RMS, nv.FLT_EPS, 0.5, M, T, H)

    @add("qkv_prep_bwd", "hbm", M * d * (2 * 2 + 4 + 4 + 4 + 2 + 2 * 2))
    def _():
        qkv, dq, dk, dqn, dgp = rb(M, 3 * d), rf(M, d), rf(M, d), rf(M, d), rb(M, d)
        dqkv, dbg = torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16), torch.zeros(64, device=dev)
        return lambda: nv.qkv_prep_bwd(qkv, dq, dk, dqn, dgp, dqkv, inv_freq, nv.NORM_RMS, nv.FLT_EPS, 0.5, M, T,
                                       H, dbg=dbg)

    @add("attn_bwd_prep", "hbm", M * d * (2 + 2 + 2 + 2 + 2 + 4) + B * H * T * 4)
    def _():
        dog, o, gate = rb(M, d), rb(M, d), torch.sigmoid(rf(M, d)).bfloat16()
        do, dgate = torch.empty_like(o), torch.empty_like(o)
        D, dq = torch.empty(B, H, T, device=dev), torch.empty(M, d, device=dev)
        return lambda: nv.attn_bwd_prep(dog, o, gate, do, dgate, D, B, T, H, dq_zero=dq)

    @add("cross_entropy", "hbm", M * V * (2 + 2))
    def _():
        logits = rb(M, V)
        labels = torch.randint(0, V, (M,), device=dev, generator=g)
        rows, sb, lo = torch.empty(M, device=dev), torch.empty(4, device=dev), torch.empty(1, device=dev)
        return lambda: nv.cross_entropy(logits, labels, loss_rows=rows, scale_buf=sb, loss_out=lo, write_grad=True)

    @add("embedding_fwd", "hbm", M * (d * 4 * 2 + 8))
    def _():
        ids = torch.randint(0, V, (M,), device=dev, generator=g)
        emb, x = rf(V, d) * 0.02, torch.empty(M, d, device=dev)
        return lambda: nv.embedding_fwd(ids, emb, x)

    n_adam = 2 * V * d + 17 * d + 8 * 64

    @add("adamw", "hbm", n_adam * 28 + V * d * 2)
    def _():
        big = [torch.nn.Parameter(rf(V, d) * 0.02), torch.nn.Parameter(rf(V, d) * 0.02)]
        vecs = [torch.nn.Parameter(torch.zeros(d, device=dev)) for _ in range(17)] + \
               [torch.nn.Parameter(torch.zeros(64, device=dev)) for _ in range(8)]
        for p in big + vecs:
            p.grad = rf(*p.shape) * 1e-3
        big[1]._rgpt_shadow = torch.empty(V, d, device=dev, dtype=torch.bfloat16)  # the lm_head's GEMM copy
        opt = Muon([{"params": big[1:], "use_muon": False, "weight_decay": 0.1},
                    {"params": big[:1] + vecs, "use_muon": False, "weight_decay": 0.0}], lr=6e-4)
        opt.concurrent = False
        return opt.step

    L = 8
    ns_flops = L * (4 * 5 * (2 * d ** 3 * 3) + 2 * 5 * (2 * d * d * 4 * d * 2 + 2 * d ** 3) + 5 * (2 * 64 ** 3 * 3))

    @add("muon_newton_schulz", "tensor", ns_flops)
    def _():
        mats = [torch.nn.Parameter(rf(*s) * 0.02) for _ in range(L)
                for s in [(d, d)] * 4 + [(4 * d, d), (d, 4 * d), (64, 64)]]
        for p in mats:
            p.grad = rf(*p.shape) * 1e-3
        opt = Muon([{"params": mats, "use_muon": True}], lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
        opt.concurrent = False
        return opt.step

    def ns_case(n, xr, xc):
        from rgpt_b200.optimizer import _NSWorkspace, newton_schulz_batched

        ws = _NSWorkspace(n, xr, xc, dev)
        x = rf(n, xr, xc)
        ws.X[:, :xr, :xc].copy_((x / x.flatten(1).norm(dim=1)[:, None, None]).bfloat16())
        return lambda: newton_schulz_batched(ws, 5)

    for n_, xr_, xc_ in ((32, d, d), (16, d, 4 * d), (8, 64, 64), (1, d, 4 * d)):
        add(f"ns_{n_}x{xr_}x{xc_}", "tensor", n_ * 5 * (2.0 * xr_ * xr_ * xc_ * 2 + 2.0 * xr_ ** 3))(
            lambda n_=n_, xr_=xr_, xc_=xc_: ns_case(n_, xr_, xc_))

    @add("attn_drop_mask", "alu", B * H * T * T / 2)
    def _():
        seed = torch.tensor([12345], dtype=torch.int64, device=dev)
        drop = nv.Drop(torch.empty(B * H, T // 32, T, device=dev, dtype=torch.int32), seed, 2, 0.1)
        return lambda: nv.attn_drop_mask(drop, B, T, H)

    return cases


def run_kernels(args):
    dev, _ = _cuda_device()
    peaks = load_peaks()
    flush = L2Flush(dev)
    out = {}
    for name, bound, work, setup in kernel_cases(dev):
        if args.only and name not in args.only.split(","):
            continue
        fn = setup()
        ms = time_launches(fn, args.launches, flush)
        if bound == "tensor":
            ach, unit, peak = work / (ms * 1e-3) / 1e12, "TFLOP/s", peaks["bf16_tflops"]
        elif bound == "hbm":
            ach, unit, peak = work / (ms * 1e-3) / 1e9, "GB/s", peaks["hbm_gbs"]
        else:
            ach, unit, peak = work / (ms * 1e-3) / 1e9, "G elements/s", None
        out[name] = {"us": round(ms * 1e3, 1), "bound": bound, "achieved": round(ach, 1), "unit": unit,
                     "frac": round(ach / peak, 3) if peak else None,
                     "work": work, "work_unit": "FLOP" if bound == "tensor" else ("bytes" if bound == "hbm"
                                                                                  else "elements")}
        del fn
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "single-launch kernel times (gpt-small sizes)", "unit": "us", "n_gpus": 1,
                      "method": "median CUDA-event time of each launch after an L2 flush (256 MB write, then 256 MB read: L2 clean and cold)",
                      "peaks": {"bf16_tflops": peaks["bf16_tflops"], "hbm_gbs": peaks["hbm_gbs"],
                                "source": peaks["source"]},
                      "kernels": out}), flush=True)


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


def cpu_train_baseline(cfg, T, budget_s=30.0):
    threads = os.cpu_count() or 1
    times = _cpu_train_steps(cfg, T, 1, threads)  # warm-up step, also sizes the sample
    n = max(1, min(5, int(budget_s / max(times[0], 1e-3))))
    times = _cpu_train_steps(cfg, T, n, threads)
    per_step = statistics.median(times)
    return {"value": round(T / per_step, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} oracle training steps (forward, CE, backward, Muon+AdamW, dropout "
                      f"{cfg['dropout']} from torch's generator) on 1 sequence x {T} tokens, "
                      f"fp32 CPU, median step {per_step:.2f} s"}


def _cpu_muon_times(n, threads):
    from oracle import ref_ops as O

    torch.set_num_threads(threads)
    c = MUON_SINGLE
    W, G, p, gp = _muon_inputs()
    mom = torch.zeros_like(W, dtype=torch.bfloat16)
    m1, v1 = torch.zeros_like(p), torch.zeros_like(p)
    R, C = c["shape"]
    times = []
    for i in range(n):
        t0 = time.perf_counter()
        upd = O.muon_update(G, mom, c["momentum"], c["ns_steps"], True, O.muon_scale(R, C))
        W.add_(upd.float(), alpha=-c["lr"])
        O.adamw_step([p], [gp], [m1], [v1], i + 1, c["lr"], 0.0, 0.9, 0.95, 1e-8)
        times.append(time.perf_counter() - t0)
    return times


def cpu_muon_baseline(budget_s=10.0):
    threads = os.cpu_count() or 1
    t = _cpu_muon_times(2, threads)
    n = max(3, min(50, int(budget_s / max(t[-1], 1e-4))))
    times = _cpu_muon_times(n, threads)
    ms = 1e3 * statistics.median(times)
    return {"value": round(ms, 3), "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"median of {n} oracle Muon steps (muon_update in bf16 + p.add_ + AdamW on the 512-vector), "
                      f"fp32/bf16 CPU"}


def _cpu_ffn_tflops(M, n, threads):
    from oracle import ref_ops as O

    torch.set_num_threads(threads)
    K, N = FFN_SWEEP["K"], FFN_SWEEP["N"]
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g)
    w1 = torch.randn(N, K, generator=g) * FFN_SWEEP["w_std"]
    w2 = torch.randn(N, K, generator=g) * FFN_SWEEP["w_std"]
    dy = torch.randn(M, K, generator=g)
    times = []
    for _ in range(n):
        t0 = time.perf_counter()
        y, pre, post = O.linear_act_forward(x, w1, w2, "squared_relu")
        O.linear_act_backward(dy, x, w1, w2, pre, post, "squared_relu")
        times.append(time.perf_counter() - t0)
    return 12.0 * M * K * N / statistics.median(times) / 1e12, statistics.median(times)


def cpu_ffn_baseline(budget_s=15.0):
    threads = os.cpu_count() or 1
    M = FFN_SWEEP["M"][0]
    _, t = _cpu_ffn_tflops(M, 1, threads)
    n = max(1, min(5, int(budget_s / max(t, 1e-3))))
    tf, t = _cpu_ffn_tflops(M, n, threads)
    return {"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"median of {n} fp32 CPU forward+backward passes of the oracle's linear+activation "
                      f"(the reference kernel file's torch composite), M={M}, squared_relu, {t:.2f} s each"}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    common = {"impl": "reference", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
              "warmup": args.warmup, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
              "data": "synthetic (seeded), as our arm"}
    if args.workload == "muon-step":
        _cpu_muon_times(max(1, args.warmup), threads)
        ms = 1e3 * statistics.mean(_cpu_muon_times(args.steps, threads))
        res = dict(common, metric="NorMuon step ms", value=round(ms, 3), unit="ms", ms_per_step=round(ms, 3),
                   higher_is_better=False, config={"workload": "muon-step", "shape": list(MUON_SINGLE["shape"]),
                                                   "parallelism": "cpu"},
                   cpu_baseline={"value": round(ms, 3), "unit": "ms", "cores": threads, "kind": "port",
                                 "sample": f"{args.steps} oracle Muon steps (all host threads)"},
                   e2e={"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    elif args.workload == "ffn-sweep":
        M = FFN_SWEEP["M"][0]
        _cpu_ffn_tflops(M, 1, threads)
        tf, t = _cpu_ffn_tflops(M, args.steps, threads)
        res = dict(common, metric="fused linear+act fwd+bwd TFLOP/s", value=round(tf, 4), unit="TFLOP/s",
                   ms_per_step=round(t * 1e3, 2), higher_is_better=True,
                   config={"workload": "ffn-sweep", "M": M, "note": "bounded CPU sample: the smallest M"},
                   cpu_baseline={"value": round(tf, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                 "sample": f"{args.steps} forward+backward passes at M={M}"},
                   e2e={"value": round(tf, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    elif args.workload == "kernels":
        res = dict(common, unavailable="single-kernel timings have no CPU counterpart")
    else:
        cfg, T = dict(wl["cfg"]), wl["T"]
        if args.dropout is not None:
            cfg["dropout"] = args.dropout
        _cpu_train_steps(cfg, T, max(1, min(args.warmup, 2)), threads)
        times = _cpu_train_steps(cfg, T, args.steps, threads)
        ms = 1000.0 * statistics.mean(times)
        value = T / (ms * 1e-3)
        res = dict(common, metric="train tokens/s", value=round(value, 2), unit="tokens/s", ms_per_step=round(ms, 2),
                   higher_is_better=True,
                   config={"workload": args.workload, "model": cfg["name"], "seq_len": T, "micro_batch": 1,
                           "parallelism": "cpu", "dropout": cfg["dropout"],
                           "note": "one 1024-token sequence per step (bounded CPU sample)"},
                   cpu_baseline={"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": f"{args.steps} oracle training steps on 1 x {T} tokens "
                                           "(fp32, all host threads)"},
                   e2e={"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0})
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=ALL_WORKLOADS, default="gpt-small")
    ap.add_argument("--cpu-budget", type=float, default=30.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="issue every kernel from Python (no CUDA graph)")
    ap.add_argument("--dropout", type=float, default=None,
                    help="dropout rate of the embedding, attention probabilities and residual branches "
                         "(default: the workload's)")
    ap.add_argument("--profile-region", action="store_true",
                    help="training workloads: after the warm-up, run K eager steps between cudaProfilerStart and "
                         "cudaProfilerStop and exit (for a profiler capture of exactly those steps)")
    ap.add_argument("--dp", choices=["sharded", "allreduce"], default="allreduce",
                    help="data-parallel step: sharded (bf16 gradient reduce-scatter, each rank updates what it owns, "
                         "all-gather of the updated weights) or allreduce (fp32 gradient all-reduce overlapped with "
                         "the backward, Newton-Schulz sharded by owner)")
    ap.add_argument("--only", default=None, help="kernels workload: comma-separated case names")
    ap.add_argument("--launches", type=int, default=5, help="kernels workload: timed launches per case")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours" and args.workload != "kernels":
        log("note: warm-up raised to 3 steps")
        args.warmup = 3
    wl = WORKLOADS.get(args.workload)
    if args.impl == "reference":
        run_reference(args, wl)
    elif args.workload == "muon-step":
        run_muon_step(args)
    elif args.workload == "ffn-sweep":
        run_ffn_sweep(args)
    elif args.workload == "kernels":
        run_kernels(args)
    else:
        run_train(args, wl)


if __name__ == "__main__":
    main()
