"""One training step replayed as a single CUDA graph.

A step is zero_grad -> accum x (forward + fused loss + backward) -> optimizer step, as in
trainer.py:150-175 of the reference: about 300 native kernel launches for the gpt-small
configuration, many of them a few microseconds long. Replaying them as one CUDA graph removes
the gap the GPU leaves between stream launches and the Python cost of issuing them.

What a graph fixes at capture, and how this class keeps each step correct:
  * Kernel arguments. Per-step optimizer scalars (scheduler learning rates, momentum, AdamW bias
    corrections) are read by the update kernels from a device block that the optimizer refills
    before every replay (Muon.use_device_hparams / stage_device_hparams).
  * Buffers. The token ids live in a static device buffer; every call copies its batch there
    (from pinned host memory or from the device). Activations, gradients and optimizer state
    are the engine's and optimizer's persistent buffers.
  * The loss. The returned 0-d tensor is the graph's static output: it holds the latest step's
    loss until the next call.
The first `warmup` calls run eagerly. They are real training steps, and they create the
optimizer state and descriptor tables, whose synchronous allocation and upload cannot be
captured. The next call captures the step and replays it; every later call replays.

Data-parallel steps (DistMuon under an initialised NCCL process group) are captured the same way:
the gradient-bucket all-reduces issued during the backward, the waits for them and the all-gather
of the sharded Newton-Schulz results become nodes of the graph. Every rank makes the same calls, so
every rank captures (and later replays) the same collectives in the same order. The first eager
step installs DistMuon's bucket hooks, so the captured step is the steady-state one.
"""
from __future__ import annotations

import torch

from . import _lib


def _data_parallel() -> bool:
    import torch.distributed as dist

    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


class GraphedTrainStep:
    """`step = GraphedTrainStep(model, opt, micro_batch, seq_len, accum)`, then
    `loss = step(ids)` with ids of shape [accum, micro_batch, seq_len + 1] (inputs are
    ids[..., :-1], labels ids[..., 1:]). Returns the last micro-batch's total loss."""

    def __init__(self, model, optimizer, micro_batch: int, seq_len: int, accum: int = 1, warmup: int = 2):
        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("GraphedTrainStep needs a CUDA model (there is no CPU path)")
        self.model, self.opt = model, optimizer
        self.accum, self.warmup = int(accum), int(warmup)
        self.inv_accum = 1.0 / self.accum
        self.ids = torch.empty(self.accum, micro_batch, seq_len + 1, dtype=torch.long, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches: int | None = None  # native kernels in one replay (counted at capture)
        self.calls = 0
        self._loss: torch.Tensor | None = None
        optimizer.use_device_hparams()

    def _body(self) -> torch.Tensor:
        self.opt.zero_grad(set_to_none=True)
        total = None
        for a in range(self.accum):
            total, _, _ = self.model.forward_loss(self.ids[a, :, :-1], self.ids[a, :, 1:])
            (total * self.inv_accum).backward()
        self.opt.step()
        return total

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        if tuple(ids.shape) != tuple(self.ids.shape):
            raise ValueError(f"ids must have shape {tuple(self.ids.shape)}, got {tuple(ids.shape)}")
        if ids.data_ptr() != self.ids.data_ptr():
            self.ids.copy_(ids, non_blocking=True)
        # parameters changed outside the optimizer kernels (a checkpoint load, a manual edit) refresh
        # their bf16 GEMM copies here: a replay does not run the engine's Python
        self.model.engine().sync_shadows()
        self.opt.stage_device_hparams()
        self.calls += 1
        if self.calls <= self.warmup:
            return self._body()
        if self.graph is None:
            g = torch.cuda.CUDAGraph()
            n0 = _lib.launch_count
            # every collective of the eager steps has completed before the capture starts; with a
            # process group, other threads' CUDA calls (the NCCL watchdog's event queries) must not
            # invalidate this thread's capture
            torch.cuda.synchronize()
            mode = "thread_local" if _data_parallel() else "global"
            with torch.cuda.graph(g, capture_error_mode=mode):
                self._loss = self._body()
            self.launches = _lib.launch_count - n0
            _lib.launch_count = n0
            self.graph = g
        self.graph.replay()
        _lib.launch_count += self.launches
        return self._loss

    def eager(self, ids: torch.Tensor) -> torch.Tensor:
        """One step issued launch by launch (same kernels and scalars as a replay), e.g. to time
        individual kernels with events."""
        if ids.data_ptr() != self.ids.data_ptr():
            self.ids.copy_(ids, non_blocking=True)
        self.opt.stage_device_hparams()
        return self._body()

    def release(self) -> None:
        """Drop the captured graph (and its memory pool); the next call captures again. A graph that
        holds collectives must be released before the process group is destroyed."""
        self.graph = None
        self._loss = None
