"""Muon / DistMuon with the reference's constructor and state layout (optimizer.py).

Every step runs on sm_100a kernels:
  * AdamW groups: one multi-tensor launch per group (rgpt_adamw), also refreshing
    the bf16 shadows the GEMMs read.
  * Muon groups: matrices are batched by shape class. Per class: one
    momentum/Nesterov/transpose kernel writes a bf16 stack X and its Frobenius
    norms, one scale kernel, then ns_steps x 3 batched tcgen05 GEMMs
        A = X X^T;  B = b*A + c*A^2 (fused epilogue);  X = a*X + B X (fused epilogue)
    and one apply kernel (weight decay, lr * multiplier, bf16 shadow).
State keys match the reference: momentum_buffer (bf16), exp_avg, exp_avg_sq and
the group counter _adam_step, so optimizer state_dicts interchange.

Names: the reference README calls these NorMuon / DistNorMuon with a
polar_express orthogonaliser; its code implements Muon / DistMuon with the
fixed quintic zeropower_via_newtonschulz5 (optimizer.py:8-45). Both names are
exported with the code's semantics; the NS coefficients are a parameter.
"""
from __future__ import annotations

import math
import os
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

from . import native as nv

NS_COEFFS = (3.4445, -4.7750, 2.0315)  # optimizer.py:19
_ADAM_CHUNK = 16384
_HP_RING = 4  # pinned host slots for the per-step scalars (copies in flight before a slot is reused)


def _muon_scale(m: int, n: int) -> float:
    """sqrt(max(1, m/n)) (optimizer.py:130-133)."""
    r = m / n
    return math.sqrt(r) if r > 1.0 else 1.0


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def trainer_param_groups(model, tie_word_embeddings=False, weight_decay=0.1):
    """The Trainer's three groups (trainer.py:66-95): Muon / AdamW-decay / AdamW-no-decay."""
    muon, dec, nodec = [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if not tie_word_embeddings and "lm_head" in name:
            dec.append(p)
        elif "emb" in name:
            nodec.append(p)
        elif p.ndim >= 2:
            muon.append(p)
        elif "norm" in name or "bias" in name:
            nodec.append(p)
        else:
            dec.append(p)
    return [
        {"params": muon, "use_muon": True},
        {"params": dec, "use_muon": False, "weight_decay": weight_decay},
        {"params": nodec, "use_muon": False, "weight_decay": 0.0},
    ]


def _table(rows: List[List[int]], device) -> torch.Tensor:
    return torch.tensor(rows, dtype=torch.int64).to(device, non_blocking=False)


# How the bf16 Newton-Schulz iteration runs: "chain" = the whole iteration of a shape class in one persistent
# kernel (rgpt_ns_chain), "batched" = 3 batched GEMM launches per step. RGPT_NS_IMPL overrides the default.
NS_IMPL = os.environ.get("RGPT_NS_IMPL", "chain")


class _NSWorkspace:
    """bf16 Newton-Schulz buffers for n matrices of one shape class (rows <= cols after transpose)."""

    def __init__(self, n, xr, xc, device):
        self.n, self.xr, self.xc = n, xr, xc
        rp, cp = _pad8(xr), _pad8(xc)
        self.X = torch.zeros(n, rp, cp, device=device, dtype=torch.bfloat16)
        self.X2 = torch.zeros_like(self.X)
        self.A = torch.zeros(n, rp, rp, device=device, dtype=torch.bfloat16)
        self.B = torch.zeros_like(self.A)
        self.sumsq = torch.zeros(n, device=device, dtype=torch.float32)
        self.ctr = torch.zeros(n * 3 * 8, device=device, dtype=torch.int32)  # the chain kernel's counters


def newton_schulz_batched(ws: _NSWorkspace, steps: int, coeffs=NS_COEFFS, impl: Optional[str] = None) -> torch.Tensor:
    """Run the quintic NS iteration in place on ws.X (already normalised); returns the result buffer."""
    a, b, c = coeffs
    if (impl or NS_IMPL) == "chain":
        if ws.ctr.numel() < ws.n * 3 * steps:
            ws.ctr = torch.zeros(ws.n * 3 * steps, device=ws.X.device, dtype=torch.int32)
        nv.ns_chain(ws.X, ws.X2, ws.A, ws.B, ws.xr, ws.xc, steps, a, b, c, ws.ctr)
        return ws.X2 if steps % 2 else ws.X
    X, X2 = ws.X, ws.X2
    for _ in range(steps):
        nv.gemm(X, X, ws.A)                                                     # A = X X^T
        nv.gemm(ws.A, ws.A, ws.B, epi=nv.EPI_POLY_BF16, alpha=c, beta=b, c=ws.A)  # B = b*A + c*A@A
        nv.gemm(ws.B, X.transpose(1, 2), X2, epi=nv.EPI_POLY_BF16, alpha=1.0, beta=a, c=X)  # X = a*X + B@X
        X, X2 = X2, X
    return X


class _NSWorkspaceF32:
    """fp32 Newton-Schulz buffers for n matrices of one shape class (rows <= cols after transpose).

    X, A, Bm hold the fp32 iterates. The bf16 operand stacks carry each fp32 value as hi + lo
    (hi = bf16(v), lo = bf16(v - hi)), blocks stacked along the GEMM's K so that one bf16 GEMM sums
    hi*hi + hi*lo + lo*hi:
      WX  [rp, 4cp] = [Xh | Xh | Xl | Xh]: A-operand columns [0, 3cp), B-operand columns [cp, 4cp)
      WA  [rp, 4rp] = [Ah | Ah | Al | Ah]: the same pairing for A @ A (A is symmetric)
      WB  [rp, 3rp] = [Bh | Bh | Bl]     : A operand of B @ X
      WXr [3rp, cp] = [Xh ; Xl ; Xh]     : B operand of B @ X, read MN-major (K runs down the rows)
    Padding stays zero, so the padded rows/columns of every product are zero too."""

    def __init__(self, n, xr, xc, device):
        self.n, self.xr, self.xc = n, xr, xc
        rp, cp = _pad8(xr), _pad8(xc)
        self.rp, self.cp = rp, cp
        f32, bf = dict(device=device, dtype=torch.float32), dict(device=device, dtype=torch.bfloat16)
        self.X, self.X2 = torch.zeros(n, rp, cp, **f32), torch.zeros(n, rp, cp, **f32)
        self.A, self.Bm = torch.zeros(n, rp, rp, **f32), torch.zeros(n, rp, rp, **f32)
        self.WX = torch.zeros(n, rp, 4 * cp, **bf)
        self.WXr = torch.zeros(n, 3 * rp, cp, **bf)
        self.WA = torch.zeros(n, rp, 4 * rp, **bf)
        self.WB = torch.zeros(n, rp, 3 * rp, **bf)
        self.sumsq = torch.zeros(n, **f32)


def newton_schulz_batched_f32(ws: _NSWorkspaceF32, steps: int, coeffs=NS_COEFFS) -> torch.Tensor:
    """The quintic NS iteration at fp32 accuracy on ws.X (already normalised); returns the result buffer.

    Per step: A = X X^T (fp32 out); B = b*A + c*A@A (POLY_F32); X = a*X + B@X (POLY_F32), each product
    one tcgen05 bf16 GEMM over K tripled (hi/lo operand blocks), fp32 accumulation."""
    a, b, c = coeffs
    xr, xc, rp, cp = ws.xr, ws.xc, ws.rp, ws.cp
    X, X2 = ws.X, ws.X2
    for _ in range(steps):
        nv.ns_split(X[:, :xr, :xc], dst=ws.WX[:, :xr, :xc], nblk=4, blk_off=cp, lo_mask=0b0100)
        nv.ns_split(X[:, :xr, :xc], dst=ws.WXr[:, :xr, :xc], nblk=3, blk_off=rp * cp, lo_mask=0b010)
        nv.gemm(ws.WX[:, :, :3 * cp], ws.WX[:, :, cp:], ws.A, epi=nv.EPI_STORE_F32)               # A = X X^T
        nv.ns_split(ws.A[:, :xr, :xr], dst=ws.WA[:, :xr, :xr], nblk=4, blk_off=rp, lo_mask=0b0100)
        nv.gemm(ws.WA[:, :, :3 * rp], ws.WA[:, :, rp:], ws.Bm, epi=nv.EPI_POLY_F32, alpha=c, beta=b,
                c=ws.A)                                                                          # B = b*A + c*A@A
        nv.ns_split(ws.Bm[:, :xr, :xr], dst=ws.WB[:, :xr, :xr], nblk=3, blk_off=rp, lo_mask=0b100)
        nv.gemm(ws.WB, ws.WXr.transpose(1, 2), X2, epi=nv.EPI_POLY_F32, alpha=1.0, beta=a, c=X)  # X = a*X + B@X
        X, X2 = X2, X
    return X


class _NSView:
    """The NS buffers of matrices [s, e) of a shape-class workspace (contiguous along the batch)."""

    def __init__(self, ws: _NSWorkspace, s: int, e: int):
        self.n, self.xr, self.xc = e - s, ws.xr, ws.xc
        self.X, self.X2, self.A, self.B = ws.X[s:e], ws.X2[s:e], ws.A[s:e], ws.B[s:e]
        self.sumsq = ws.sumsq[s:e]
        self.ctr = ws.ctr


def assign_ns_owners(shapes: List[Tuple[int, int]], world: int) -> List[int]:
    """Owner rank of each Muon matrix's Newton-Schulz iteration, balanced by NS FLOPs.

    `shapes` are the (rows, cols) each matrix has after the rows <= cols transpose. Greedy
    longest-processing-time assignment (heaviest matrices first, to the least loaded rank, lowest
    rank on ties); deterministic, so every rank computes the same assignment."""
    cost = [2 * r * r * c * 2 + 2 * r ** 3 for r, c in shapes]
    order = sorted(range(len(shapes)), key=lambda i: (-cost[i], i))
    load = [0] * world
    owner = [0] * len(shapes)
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += cost[i]
    return owner


def _slot(n: int, a: int = 8) -> int:
    return (n + a - 1) // a * a


class ShardLayout:
    """Which rank updates what in the sharded data-parallel step, and where it sits in a packed buffer.

    Rank r owns elements [r*S, (r+1)*S) of the flat AdamW space (every AdamW tensor of every group, in
    group order, each starting on an 8-element boundary) and the Muon matrices that assign_ns_owners
    gives it (whole matrices: Newton-Schulz needs all of one). A packed buffer is `world` chunks of C
    elements; rank r's chunk holds its AdamW slice at [0, S) and its Muon matrices from S on. Gradients
    travel in this layout through one reduce-scatter (rank r receives chunk r, summed over ranks) and
    updated parameters through one all-gather (every rank receives every chunk)."""

    def __init__(self, muon: List[torch.Tensor], adam: List[Tuple[int, torch.Tensor]], world: int):
        self.world = world
        self.adam = []  # (group index, param, flat start)
        off = 0
        for gi, p in adam:
            self.adam.append((gi, p, off))
            off += _slot(p.numel())
        self.adam_total = off
        self.S = _slot(-(-off // world)) if off else 0
        shapes = []
        for p in muon:
            R, C = p.shape[0], p.numel() // p.shape[0]
            shapes.append((C, R) if R > C else (R, C))
        owners = assign_ns_owners(shapes, world) if muon else []
        used = [self.S] * world
        self.muon = []  # (param, owner, offset in the owner's chunk)
        for p, o in zip(muon, owners):
            self.muon.append((p, o, used[o]))
            used[o] += _slot(p.numel())
        self.C = _slot(max(used)) if used else 0

    def owned_muon(self, r: int) -> List[torch.Tensor]:
        return [p for p, o, _ in self.muon if o == r]

    def adam_slices(self, r: int):
        """(group, param, lo, hi, flat start) of every AdamW element range rank r owns."""
        a, b = r * self.S, (r + 1) * self.S
        out = []
        for gi, p, f0 in self.adam:
            lo, hi = max(a, f0), min(b, f0 + p.numel())
            if lo < hi:
                out.append((gi, p, lo - f0, hi - f0, f0))
        return out

    def segments(self, ranks, tensor_of, second_of=None, base_of=None):
        """(tensor, bf16 copy or None, buffer offset, element offset, count) of the chunks of `ranks`;
        tensor_of(param) gives the tensor a segment reads or writes (None: skipped); base_of(rank) the
        buffer offset of the rank's chunk (default rank * C)."""
        segs = []
        for r in ranks:
            base = r * self.C if base_of is None else base_of(r)
            for gi, p, lo, hi, f0 in self.adam_slices(r):
                t = tensor_of(p)
                if t is not None:
                    segs.append((t, second_of(p) if second_of else None, base + f0 + lo - r * self.S, lo, hi - lo))
            for p, o, off in self.muon:
                if o == r:
                    t = tensor_of(p)
                    if t is not None:
                        segs.append((t, second_of(p) if second_of else None, base + off, 0, p.numel()))
        return segs


def _muon_rows(params, grads, moms) -> List[List[int]]:
    rows = []
    for p, g, m in zip(params, grads, moms):
        sh = getattr(p, "_rgpt_shadow", None)
        rows.append([p.data_ptr(), g.data_ptr(), m.data_ptr(), sh.data_ptr() if sh is not None else 0])
    return rows


class Muon(torch.optim.Optimizer):
    """Muon for 2-D weights (group use_muon=True) + AdamW for the rest (optimizer.py:143-272)."""

    def __init__(self, params: List[Dict[str, Any]], lr: float = 3e-4, weight_decay: float = 0.01,
                 momentum: float = 0.95, nesterov: bool = True, adam_betas: Tuple[float, float] = (0.9, 0.95),
                 adam_eps: float = 1e-8, muon_lr_multiplier: float = 100.0, ns_steps: int = 5,
                 ns_coeffs: Tuple[float, float, float] = NS_COEFFS, ns_precision: str = "bf16"):
        """ns_precision: "bf16" iterates Newton-Schulz in bf16 as the reference does (optimizer.py:20-44);
        "fp32" iterates it at fp32 accuracy (hi/lo bf16 operands, fp32 accumulation) from the same bf16
        input, the update still rounded to bf16 as the reference rounds it (optimizer.py:68)."""
        if ns_precision not in ("bf16", "fp32"):
            raise ValueError(f"ns_precision must be 'bf16' or 'fp32', got {ns_precision!r}")
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                        adam_betas=adam_betas, adam_eps=adam_eps, muon_lr_multiplier=muon_lr_multiplier,
                        ns_steps=ns_steps, ns_coeffs=tuple(ns_coeffs), ns_precision=ns_precision)
        super().__init__(params, defaults)
        self._cache: Dict[Any, Any] = {}
        self._hp_dev: Optional[torch.Tensor] = None
        # Independent update jobs (each Newton-Schulz shape class, each AdamW group) run on their own
        # CUDA streams, forked from and joined back into the caller's stream (inside a captured step
        # too), so the HBM-bound AdamW overlaps the small Newton-Schulz GEMMs and the shape classes
        # overlap each other's tails. Set to False to issue everything on the caller's stream.
        self.concurrent = True
        self._streams: List[torch.cuda.Stream] = []

    # ------------------------------------------------------------------ device scalars
    def use_device_hparams(self) -> None:
        """Make the update kernels read each step's scalars (learning rates, momentum, betas, AdamW
        bias corrections) from a device block that stage_device_hparams() refills, instead of
        kernel arguments. A captured CUDA graph of the step needs this: its kernel arguments are
        frozen at capture, the block's contents are not. Call stage_device_hparams() before
        every step from then on."""
        if self._hp_dev is not None:
            return
        dev = next(p.device for g in self.param_groups for p in g["params"])
        n = len(self.param_groups) * nv.HP_FLOATS
        self._hp_dev = torch.zeros(n, device=dev, dtype=torch.float32)
        self._hp_host = [torch.zeros(n, dtype=torch.float32).pin_memory() for _ in range(_HP_RING)]
        self._hp_done: List[Optional[torch.cuda.Event]] = [None] * _HP_RING
        self._hp_slot = 0

    def stage_device_hparams(self) -> None:
        """Compute the next step's per-group scalars on the host (advancing the AdamW step
        counters) and enqueue their copy into the device block on the current stream. The values
        are rounded exactly as the by-value path rounds them, so both paths update identically."""
        if self._hp_dev is None:
            raise RuntimeError("stage_device_hparams() needs use_device_hparams() first")
        slot = self._hp_slot
        if self._hp_done[slot] is not None:
            self._hp_done[slot].synchronize()  # the copy that last read this pinned slot has run
        buf = self._hp_host[slot]
        v = buf.numpy()
        v[:] = 0.0
        f32 = np.float32
        for gi, group in enumerate(self.param_groups):
            o = gi * nv.HP_FLOATS
            lr, wd = float(group["lr"]), float(group["weight_decay"])
            if group.get("use_muon", False):
                muon_lr = lr * float(group["muon_lr_multiplier"])
                v[o] = f32(group["momentum"])
                v[o + 1] = f32(1.0) - f32(lr) * f32(wd)  # rgpt_muon_apply's float 1 - lr*wd
                v[o + 2] = -f32(muon_lr)
            else:
                beta1, beta2 = group["adam_betas"]
                step_i = int(group.get("_adam_step", 0)) + 1
                group["_adam_step"] = step_i
                b1, b2 = float(f32(beta1)), float(f32(beta2))
                bc1 = 1.0 - b1 ** step_i  # rgpt_adamw: double pow of the float betas
                bc2 = 1.0 - b2 ** step_i
                v[o:o + 7] = [f32(lr), f32(wd), f32(b1), f32(b2), f32(group["adam_eps"]), f32(1.0 / bc1),
                              f32(1.0 / math.sqrt(bc2))]
        self._hp_dev.copy_(buf, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._hp_done[slot] = ev
        self._hp_slot = (slot + 1) % _HP_RING

    def _hp(self, gi: int) -> Optional[int]:
        """Device address of group gi's scalar block, or None on the by-value path."""
        if self._hp_dev is None:
            return None
        return self._hp_dev.data_ptr() + gi * nv.HP_FLOATS * 4

    # ------------------------------------------------------------------ state
    def load_state_dict(self, state_dict):
        """torch's loader casts every state tensor to its parameter's dtype, which would turn the bf16
        momentum buffers into fp32. Restore the kernels' dtypes (momentum_buffer bf16, AdamW moments
        fp32), and copy into the state tensors that already exist: their addresses are baked into the
        update kernels' descriptor tables and into captured CUDA graphs of the step."""
        before = {p: dict(st) for p, st in self.state.items()}
        super().load_state_dict(state_dict)
        with torch.no_grad():
            for p, st in self.state.items():
                for k, v in list(st.items()):
                    if not torch.is_tensor(v) or not v.is_floating_point():
                        continue
                    want = torch.bfloat16 if k == "momentum_buffer" else torch.float32
                    old = before.get(p, {}).get(k)
                    if old is not None and old.shape == v.shape and old.dtype == want:
                        old.copy_(v)
                        st[k] = old
                    else:
                        st[k] = v.to(want).contiguous()

    # ------------------------------------------------------------------ grads
    @torch.no_grad()
    def zero_grad(self, set_to_none: bool = True):
        """Gradients that live in a model's native gradient arena are zeroed in place (their
        storage is what the backward kernels accumulate into); others follow torch semantics."""
        arenas = {}
        for group in self.param_groups:
            for p in group["params"]:
                arena = getattr(p, "_rgpt_grad_arena", None)
                if arena is not None and p.grad is not None:
                    arenas[id(arena)] = arena
                elif p.grad is not None:
                    if set_to_none:
                        p.grad = None
                    else:
                        p.grad.zero_()
        for a in arenas.values():
            a.zero_()

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure: Optional[Any] = None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        jobs = []
        for gi, group in enumerate(self.param_groups):
            ps = [p for p in group["params"] if p.grad is not None]
            if group.get("use_muon", False):
                jobs += self._muon_jobs(gi, group, ps)
            else:
                jobs += self._adamw_jobs(gi, group, ps)
        self._run_jobs(jobs)
        return loss

    def _run_jobs(self, jobs) -> None:
        """Run the launch-only closures: the first on the current stream, the others each on a
        side stream that waits for the current stream first and is waited for at the end."""
        if len(jobs) <= 1 or not self.concurrent:
            for job in jobs:
                job()
            return
        main = torch.cuda.current_stream()
        while len(self._streams) < len(jobs) - 1:
            self._streams.append(torch.cuda.Stream(device=main.device))
        side = self._streams[:len(jobs) - 1]
        for st in side:
            st.wait_stream(main)
        for job, st in zip(jobs[1:], side):
            with torch.cuda.stream(st):
                job()
        jobs[0]()
        for st in side:
            main.wait_stream(st)

    def _muon_group(self, gi, group, params):
        """Plan and run one Muon group on the current stream."""
        for job in self._muon_jobs(gi, group, params):
            job()

    def _muon_jobs(self, gi, group, params):
        """Per Newton-Schulz shape class, a closure that launches its kernels. State, descriptor
        tables and workspaces are created here, on the caller's stream."""
        if not params:
            return []
        lr = float(group["lr"])
        wd = float(group["weight_decay"])
        muon_lr = lr * float(group["muon_lr_multiplier"])
        beta = float(group["momentum"])
        nesterov = bool(group["nesterov"])
        steps = int(group.get("ns_steps", 5))
        coeffs = tuple(group.get("ns_coeffs", NS_COEFFS))
        fp32 = group.get("ns_precision", "bf16") == "fp32"
        # batch by the shape Newton-Schulz sees (rows <= cols after transposing), so e.g. fc1 [4d, d]
        # and fc2 [d, 4d] share one stack; prep/apply run per original shape on slices of it
        classes: Dict[Tuple[int, int], Dict[Tuple[int, int], List[torch.Tensor]]] = {}
        for p in params:
            st = self.state[p]
            if len(st) == 0:
                st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
            R, C = p.shape[0], p.numel() // p.shape[0]
            xr, xc = (C, R) if R > C else (R, C)
            classes.setdefault((xr, xc), {}).setdefault((R, C), []).append(p)
        jobs = []
        for (xr, xc), subs in classes.items():
            ordered = [(rc, ps) for rc, ps in sorted(subs.items())]
            all_ps = [p for _, ps in ordered for p in ps]
            rows_all = _muon_rows(all_ps, [p.grad for p in all_ps], [self.state[p]["momentum_buffer"] for p in all_ps])
            key = ("muon", gi, xr, xc, fp32, tuple(r[0] for r in rows_all), tuple(r[1] for r in rows_all))
            ent = self._cache.get(key)
            if ent is None:
                dev = all_ps[0].device
                tables, off = [], 0
                for (R, C), ps in ordered:
                    tables.append((R, C, off, len(ps), _table(rows_all[off:off + len(ps)], dev)))
                    off += len(ps)
                ent = (tables, _NSWorkspace(len(all_ps), xr, xc, dev),
                       _NSWorkspaceF32(len(all_ps), xr, xc, dev) if fp32 else None)
                self._cache[key] = ent
            tables, ws, ws32 = ent

            def run(tables=tables, ws=ws, ws32=ws32):
                ws.sumsq.zero_()
                for R, C, off, n, table in tables:
                    nv.muon_prep(table, n, R, C, ws.X[off:off + n], beta, nesterov, ws.sumsq[off:off + n],
                                 hp=self._hp(gi))
                if ws32 is None:
                    nv.ns_scale(ws.X, ws.xr, _pad8(ws.xc), ws.n, ws.sumsq)
                    out = newton_schulz_batched(ws, steps, coeffs)
                else:
                    # the bf16 Nesterov stack, normalised into fp32, iterated at fp32 accuracy, and the
                    # result written back as bf16 (one hi block) for the apply kernel
                    r_, c_ = ws.xr, ws.xc  # this class's shape (the loop variables move on before jobs run)
                    nv.ns_split(ws.X[:, :r_, :c_], sumsq=ws.sumsq, xout=ws32.X[:, :r_, :c_])
                    res = newton_schulz_batched_f32(ws32, steps, coeffs)
                    nv.ns_split(res[:, :r_, :c_], dst=ws.X[:, :r_, :c_], nblk=1, blk_off=0, lo_mask=0)
                    out = ws.X
                for R, C, off, n, table in tables:
                    nv.muon_apply(table, n, R, C, out[off:off + n], lr, wd, muon_lr, _muon_scale(R, C),
                                  hp=self._hp(gi))
            jobs.append(run)
        return jobs

    def _adamw_group(self, gi, group, params):
        """Plan and run one AdamW group on the current stream."""
        for job in self._adamw_jobs(gi, group, params):
            job()

    def _adamw_jobs(self, gi, group, params, slices=None):
        """A closure launching the group's multi-tensor AdamW kernel (the step counter and the
        optimizer state are advanced / created here, on the caller's stream). slices: optional
        (param, lo, hi) element ranges to update instead of whole parameters (the sharded step); the
        counter advances even when the list is empty, so every rank keeps the same step."""
        if slices is not None:
            params = list(dict.fromkeys(p for p, _, _ in slices))
        elif not params:
            return []
        lr = float(group["lr"])
        wd = float(group["weight_decay"])
        beta1, beta2 = group["adam_betas"]
        eps = float(group["adam_eps"])
        step_i = int(group.get("_adam_step", 0))
        if self._hp_dev is None:  # else stage_device_hparams() advanced it
            step_i += 1
            group["_adam_step"] = step_i
        if not params:
            return []
        for p in params:
            st = self.state[p]
            if len(st) == 0:
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
        ranges = slices if slices is not None else [(p, 0, p.numel()) for p in params]
        rows = []
        for p, lo, hi in ranges:
            st = self.state[p]
            sh = getattr(p, "_rgpt_shadow", None)
            rows.append([p.data_ptr() + 4 * lo, p.grad.data_ptr() + 4 * lo, st["exp_avg"].data_ptr() + 4 * lo,
                         st["exp_avg_sq"].data_ptr() + 4 * lo, sh.data_ptr() + 2 * lo if sh is not None else 0,
                         hi - lo])
        key = ("adamw", gi, tuple(tuple(r) for r in rows))
        ent = self._cache.get(key)
        if ent is None:
            ct, cs = [], []
            for ti, (_, lo, hi) in enumerate(ranges):
                for s in range(0, hi - lo, _ADAM_CHUNK):
                    ct.append(ti)
                    cs.append(s)
            dev = params[0].device
            ent = (_table(rows, dev), torch.tensor(ct, dtype=torch.int32).to(dev),
                   torch.tensor(cs, dtype=torch.int64).to(dev))
            self._cache[key] = ent
        table, ct, cs = ent
        return [lambda: nv.adamw(table, ct, cs, _ADAM_CHUNK, lr, wd, float(beta1), float(beta2), eps, step_i,
                                 hp=self._hp(gi))]


class DistMuon(Muon):
    """Data-parallel Muon (optimizer.py:278-415).

    The reference wraps the model in DDP (an fp32 all-reduce of every gradient) and repeats the whole
    update on every rank. Here the model is not wrapped; this optimizer moves the data itself, in one of
    two ways:

    sharded_state=True: each rank owns part of the update (ShardLayout): whole Muon matrices,
      balanced by Newton-Schulz FLOPs, and an equal slice of every AdamW element. Per step:
        1. the gradients, packed owner-major in `reduce_dtype` (bf16 by default), go through ONE
           reduce-scatter (average over ranks): each rank receives the averaged gradients of what it owns;
        2. each rank runs momentum + Newton-Schulz + apply on its own matrices and AdamW on its own slices,
           and keeps optimizer state current only there (momentum buffers exist only for its matrices);
        3. the updated fp32 parameters go through ONE all-gather, and every rank rewrites its parameters
           and their bf16 GEMM copies from it.
      consolidate_state_dict() (a collective) gathers the full state, e.g. before a checkpoint.
    sharded_state=False (default): an fp32 all-reduce (average) of the gradient arena, bucket by bucket as the
      native backward finishes each layer, then momentum and AdamW on every rank with each Newton-Schulz
      run by one owner rank and its bf16 result all-gathered (shard_ns=False: repeated on every rank)."""

    def __init__(self, params, *args, process_group=None, shard_ns: bool = True, overlap_grad_sync: bool = True,
                 sharded_state: bool = False, reduce_dtype: torch.dtype = torch.bfloat16, **kwargs):
        super().__init__(params, *args, **kwargs)
        self.process_group = process_group
        self.shard_ns = shard_ns
        self.overlap_grad_sync = overlap_grad_sync
        self.sharded_state = sharded_state
        if reduce_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("reduce_dtype must be torch.bfloat16 or torch.float32")
        self.reduce_dtype = reduce_dtype
        self._pending: List[Any] = []    # async all-reduces launched during the backward
        self._synced: Dict[int, bool] = {}  # arena id -> every bucket reduced in the latest backward
        self._layout_cache: Dict[Any, Any] = {}

    # -- gradient-bucket hooks called by the native backward (see Engine.backward) --
    def begin(self, arena):
        self._synced[id(arena)] = False

    def ready(self, arena, start: int, end: int):
        # the collective waits for the kernels already queued on the current stream, then runs
        # alongside the rest of the backward; AVG averages over the ranks like the reference's DDP
        self._pending.append((dist.all_reduce(arena[start:end], op=dist.ReduceOp.AVG, group=self.process_group,
                                              async_op=True), arena, start, end))

    def end(self, arena):
        self._synced[id(arena)] = True

    def _world(self) -> int:
        return dist.get_world_size(self.process_group) if dist.is_available() and dist.is_initialized() else 1

    @torch.no_grad()
    def step(self, closure: Optional[Any] = None):
        world = self._world()
        if world <= 1:
            return super().step(closure)
        fp32_ns = any(g.get("ns_precision", "bf16") == "fp32" for g in self.param_groups)
        if self.sharded_state and not fp32_ns:
            loss = None
            if closure is not None:
                with torch.enable_grad():
                    loss = closure()
            self._sharded_step(dist.get_rank(self.process_group), world)
            return loss
        if not self.shard_ns or fp32_ns:
            self._average_grads()
            return super().step(closure)  # the fp32 iteration runs replicated on every rank
        # The last gradient bucket (the embedding's, finished by the last kernel of the backward) holds no
        # Muon matrix, so its all-reduce keeps running under the Newton-Schulz work and is only waited for
        # before AdamW.
        deferred = self._average_grads(defer_last=True)
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        rank = dist.get_rank(self.process_group)
        for gi, group in enumerate(self.param_groups):
            if group.get("use_muon", False):
                self._muon_group_sharded(gi, group, [p for p in group["params"] if p.grad is not None], rank, world)
        if deferred is not None:
            deferred.wait()
        for gi, group in enumerate(self.param_groups):
            if not group.get("use_muon", False):
                self._adamw_group(gi, group, [p for p in group["params"] if p.grad is not None])
        return loss

    # ------------------------------------------------------------------ sharded-state step
    def layout(self, world: int) -> "ShardLayout":
        """The ShardLayout of this optimizer's parameters that have gradients (identical on every rank)."""
        muon, adam = [], []
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                if p.grad is None:
                    continue
                if group.get("use_muon", False):
                    muon.append(p)
                else:
                    adam.append((gi, p))
        key = ("layout", world, tuple(id(p) for p in muon), tuple(id(p) for _, p in adam))
        lay = self._layout_cache.get(key)
        if lay is None:
            lay = ShardLayout(muon, adam, world)
            self._layout_cache[key] = lay
        return lay

    def _staging(self, lay: ShardLayout, rank: int, world: int):
        """Packed buffers and segment tables of the sharded step (built once per parameter/gradient set)."""
        params = [p for p, _, _ in lay.muon] + [p for _, p, _ in lay.adam]
        key = ("staging", id(lay), rank, tuple(p.data_ptr() for p in params), tuple(p.grad.data_ptr() for p in params))
        st = self._layout_cache.get(key)
        if st is not None:
            return st
        for p in params:
            if p.dtype != torch.float32 or p.grad.dtype != torch.float32 or not p.grad.is_contiguous():
                raise ValueError("the sharded step needs fp32 parameters with contiguous fp32 gradients")
        dev = params[0].device
        C = lay.C
        shadow = lambda p: getattr(p, "_rgpt_shadow", None)  # noqa: E731
        st = dict(
            send=torch.zeros(world * C, device=dev, dtype=self.reduce_dtype),
            recv=torch.zeros(C, device=dev, dtype=self.reduce_dtype),
            send32=torch.zeros(C, device=dev, dtype=torch.float32),
            recv32=torch.zeros(world * C, device=dev, dtype=torch.float32),
            # every rank's chunk of the gradients, in the owner-major layout
            pack_grads=nv.segment_table(lay.segments(range(world), lambda p: p.grad), dev),
            # the averaged gradients of what this rank owns, back into their fp32 gradient slots
            unpack_grads=nv.segment_table(lay.segments([rank], lambda p: p.grad, base_of=lambda r: 0), dev),
            # this rank's updated parameters
            pack_params=nv.segment_table(lay.segments([rank], lambda p: p, base_of=lambda r: 0), dev),
            # every rank's updated parameters, into the fp32 parameters and their bf16 GEMM copies
            unpack_params=nv.segment_table(lay.segments(range(world), lambda p: p, second_of=shadow), dev),
        )
        self._layout_cache[key] = st
        return st

    def _sharded_step(self, rank: int, world: int) -> None:
        for w, *_ in self._pending:  # hooks of an earlier all-reduce step
            w.wait()
        self._pending = []
        lay = self.layout(world)
        st = self._staging(lay, rank, world)
        pg = self.process_group
        # 1. averaged gradients of what this rank owns: pack, reduce-scatter, unpack
        nv.segment_copy(st["pack_grads"], st["send"], tensor_bf16=False)
        dist.reduce_scatter_tensor(st["recv"], st["send"], op=dist.ReduceOp.AVG, group=pg)
        nv.segment_copy(st["unpack_grads"], st["recv"], tensor_bf16=False, unpack=True)
        # 2. the update of the owned matrices and AdamW slices
        jobs = []
        owned = set(lay.owned_muon(rank))
        slices = {}
        for gi, p, lo, hi, _ in lay.adam_slices(rank):
            slices.setdefault(gi, []).append((p, lo, hi))
        for gi, group in enumerate(self.param_groups):
            if group.get("use_muon", False):
                jobs += self._muon_jobs(gi, group, [p for p in group["params"] if p in owned])
            else:
                jobs += self._adamw_jobs(gi, group, None, slices=slices.get(gi, []))
        self._run_jobs(jobs)
        # 3. every rank's updated parameters to every rank (fp32, so replicas stay identical)
        nv.segment_copy(st["pack_params"], st["send32"], tensor_bf16=False)
        dist.all_gather_into_tensor(st["recv32"], st["send32"], group=pg)
        nv.segment_copy(st["unpack_params"], st["recv32"], tensor_bf16=False, unpack=True)

    @torch.no_grad()
    def consolidate_state_dict(self) -> Dict[str, Any]:
        """Collective: give every rank the full optimizer state (each Muon matrix's momentum from its owner,
        each AdamW moment slice from its owner), then return state_dict(). Call it on every rank, e.g.
        before rank 0 writes a checkpoint."""
        world = self._world()
        if world <= 1 or not self.sharded_state:
            return self.state_dict()
        rank = dist.get_rank(self.process_group)
        lay = self.layout(world)
        dev = lay.muon[0][0].device if lay.muon else lay.adam[0][1].device
        for p, _, _ in lay.muon:
            st = self.state[p]
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
        for _, p, _ in lay.adam:
            st = self.state[p]
            if "exp_avg" not in st:
                st["exp_avg"] = torch.zeros_like(p)
                st["exp_avg_sq"] = torch.zeros_like(p)
        send = torch.zeros(lay.C, device=dev, dtype=torch.float32)
        recv = torch.zeros(world * lay.C, device=dev, dtype=torch.float32)
        keys = (("momentum_buffer", True), ("exp_avg", False), ("exp_avg_sq", False))
        for k, is_bf in keys:
            def of(p, k=k):
                return self.state[p].get(k)
            mine = nv.segment_table(lay.segments([rank], of, base_of=lambda r: 0), dev)
            allr = nv.segment_table(lay.segments(range(world), of), dev)
            # segments of one key are all bf16 (momentum) or all fp32 (moments)
            nv.segment_copy(mine, send, tensor_bf16=is_bf)
            dist.all_gather_into_tensor(recv, send, group=self.process_group)
            nv.segment_copy(allr, recv, tensor_bf16=is_bf, unpack=True)
        return self.state_dict()

    def _muon_group_sharded(self, gi, group, params, rank: int, world: int):
        if not params:
            return
        lr = float(group["lr"])
        wd = float(group["weight_decay"])
        muon_lr = lr * float(group["muon_lr_multiplier"])
        beta = float(group["momentum"])
        nesterov = bool(group["nesterov"])
        steps = int(group.get("ns_steps", 5))
        coeffs = tuple(group.get("ns_coeffs", NS_COEFFS))
        for p in params:
            st = self.state[p]
            if len(st) == 0:
                st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.bfloat16)
        rows_all = _muon_rows(params, [p.grad for p in params], [self.state[p]["momentum_buffer"] for p in params])
        key = ("muon_sharded", gi, world, rank, tuple(tuple(r) for r in rows_all))
        plan = self._cache.get(key)
        if plan is None:
            plan = self._plan_sharded(params, rows_all, world)
            self._cache[key] = plan
        for (xr, xc), cls in plan.items():
            ws = cls["ws"]
            ws.sumsq.zero_()
            # momentum (and the NS input) for every matrix: the momentum state stays replicated
            for R, C, owner, off, n, table in cls["segments"]:
                nv.muon_prep(table, n, R, C, ws.X[off:off + n], beta, nesterov, ws.sumsq[off:off + n],
                             hp=self._hp(gi))
            s, e = cls["blocks"][rank]
            send = cls["send"]
            if e > s:
                view = _NSView(ws, s, e)
                nv.ns_scale(view.X, xr, _pad8(xc), view.n, view.sumsq)
                out = newton_schulz_batched(view, steps, coeffs)
                send[:e - s].copy_(out)
            dist.all_gather_into_tensor(cls["gathered"], send, group=self.process_group)
            maxc = cls["maxc"]
            for R, C, owner, off, n, table in cls["segments"]:
                g0 = owner * maxc + (off - cls["blocks"][owner][0])
                nv.muon_apply(table, n, R, C, cls["gathered"][g0:g0 + n], lr, wd, muon_lr, _muon_scale(R, C),
                              hp=self._hp(gi))

    def _plan_sharded(self, params, rows_all, world):
        """Per shape class: matrices ordered by (owner, original shape), one prep/apply table per
        (owner, shape) run, each owner's matrices contiguous, and the all-gather buffers."""
        dev = params[0].device
        shapes = []
        for p in params:
            R, C = p.shape[0], p.numel() // p.shape[0]
            shapes.append((R, C, (C, R) if R > C else (R, C)))
        owners = assign_ns_owners([sh[2] for sh in shapes], world)
        by_class: Dict[Tuple[int, int], List[int]] = {}
        for i, sh in enumerate(shapes):
            by_class.setdefault(sh[2], []).append(i)
        plan = {}
        for (xr, xc), idx in sorted(by_class.items()):
            idx = sorted(idx, key=lambda i: (owners[i], shapes[i][0], shapes[i][1], i))
            segments, blocks, off = [], [], 0
            for r in range(world):
                start = off
                mine = [i for i in idx if owners[i] == r]
                j = 0
                while j < len(mine):
                    R, C = shapes[mine[j]][0], shapes[mine[j]][1]
                    k = j
                    while k < len(mine) and (shapes[mine[k]][0], shapes[mine[k]][1]) == (R, C):
                        k += 1
                    run = mine[j:k]
                    segments.append((R, C, r, off, len(run), _table([rows_all[i] for i in run], dev)))
                    off += len(run)
                    j = k
                blocks.append((start, off))
            maxc = max(max(e - s for s, e in blocks), 1)
            ws = _NSWorkspace(len(idx), xr, xc, dev)
            rp, cp = _pad8(xr), _pad8(xc)
            plan[(xr, xc)] = dict(ws=ws, segments=segments, blocks=blocks, maxc=maxc,
                                  send=torch.zeros(maxc, rp, cp, device=dev, dtype=torch.bfloat16),
                                  gathered=torch.zeros(world * maxc, rp, cp, device=dev, dtype=torch.bfloat16))
        return plan

    def _average_grads(self, defer_last: bool = False):
        """Finish the averaging of every gradient (waits for the bucket all-reduces issued during the
        backward, all-reduces what was not hooked). defer_last: leave the last bucket's all-reduce
        running and return its work handle, if no Muon gradient lies in that bucket."""
        ws = dist.get_world_size(self.process_group)
        pending, self._pending = self._pending, []
        deferred = None
        if defer_last and pending:
            w, arena, start, end = pending[-1]
            base = arena.data_ptr()
            muon_in = any(p.grad is not None and start <= (p.grad.data_ptr() - base) // 4 < end
                          for g in self.param_groups if g.get("use_muon", False) for p in g["params"])
            if not muon_in:
                deferred = w
                pending = pending[:-1]
        for w, *_ in pending:
            w.wait()
        nccl = dist.get_backend(self.process_group) == "nccl"
        arenas, loose = {}, []
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                a = getattr(p, "_rgpt_grad_arena", None)
                if a is not None:
                    arenas[id(a)] = a
                else:
                    loose.append(p.grad)
        for key, a in arenas.items():
            if self._synced.pop(key, False):
                continue  # every bucket was averaged during the backward
            if nccl and self.overlap_grad_sync:
                a._rgpt_sync = self  # later backwards reduce bucket by bucket
            dist.all_reduce(a, op=dist.ReduceOp.SUM, group=self.process_group)
            a.mul_(1.0 / ws)
        for g in loose:
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.process_group)
            g.mul_(1.0 / ws)
        return deferred


# Names used by the reference's README.
NorMuon = Muon
DistNorMuon = DistMuon


# ---------------------------------------------------------------------- functional API
@torch.no_grad()
def zeropower_via_newtonschulz5(G: torch.Tensor, steps: int, coeffs=NS_COEFFS, precision: str = "bf16") -> torch.Tensor:
    """Native quintic Newton-Schulz orthogonalisation of a 2-D (or batched 3-D) CUDA tensor (optimizer.py:8-45).

    precision "bf16" (the reference's): X = bf16(G), bf16 iterates; returns bf16.
    precision "fp32": X = G.float() and fp32 iterates (bf16 hi/lo operand splitting on the tensor
    cores, fp32 accumulation); returns fp32. Both return G's shape."""
    if not G.is_cuda:
        raise RuntimeError("zeropower_via_newtonschulz5 runs on CUDA tensors only (no CPU path)")
    if precision not in ("bf16", "fp32"):
        raise ValueError(f"precision must be 'bf16' or 'fp32', got {precision!r}")
    squeeze = G.dim() == 2
    Gb = G.unsqueeze(0) if squeeze else G
    n, R, C = Gb.shape
    transposed = R > C
    Xs = Gb.transpose(1, 2) if transposed else Gb
    xr, xc = Xs.shape[1], Xs.shape[2]
    if precision == "fp32":
        src = Xs if Xs.dtype in (torch.float32, torch.bfloat16) else Xs.float()
        ws = _NSWorkspaceF32(n, xr, xc, G.device)
        nv.ns_sumsq(src, ws.sumsq)
        nv.ns_split(src, sumsq=ws.sumsq, xout=ws.X[:, :xr, :xc])
        out = newton_schulz_batched_f32(ws, steps, coeffs)[:, :xr, :xc]
        out = (out.transpose(1, 2) if transposed else out).contiguous()
        return out[0] if squeeze else out
    ws = _NSWorkspace(n, xr, xc, G.device)
    ws.X[:, :xr, :xc].copy_(Xs.to(torch.bfloat16))
    ws.sumsq.copy_(ws.X.float().pow(2).sum(dim=(1, 2)))
    nv.ns_scale(ws.X, xr, _pad8(xc), n, ws.sumsq)
    out = newton_schulz_batched(ws, steps, coeffs)[:, :xr, :xc]
    out = out.transpose(1, 2) if transposed else out
    out = out.contiguous()
    return out[0] if squeeze else out


polar_express = zeropower_via_newtonschulz5


@torch.no_grad()
def muon_update(grad_2d: torch.Tensor, momentum_2d: torch.Tensor, beta: float = 0.95, ns_steps: int = 5,
                nesterov: bool = True, scale: float = 1.0) -> torch.Tensor:
    """Momentum + Nesterov + NS + scale for one matrix (optimizer.py:51-74); updates momentum in place."""
    R, C = grad_2d.shape
    dev = grad_2d.device
    g = grad_2d.float().contiguous()
    xr, xc = (C, R) if R > C else (R, C)
    ws = _NSWorkspace(1, xr, xc, dev)
    dummy = torch.zeros(R, C, device=dev, dtype=torch.float32)
    table = _table([[dummy.data_ptr(), g.data_ptr(), momentum_2d.data_ptr(), 0]], dev)
    nv.muon_prep(table, 1, R, C, ws.X, beta, nesterov, ws.sumsq)
    nv.ns_scale(ws.X, xr, _pad8(xc), 1, ws.sumsq)
    out = newton_schulz_batched(ws, ns_steps)[0, :xr, :xc]
    out = out.t() if R > C else out
    return (out.float() * scale).to(torch.bfloat16)


@torch.no_grad()
def foreach_adamw_step(params, grads, exp_avgs, exp_avg_sqs, step, lr, wd, beta1, beta2, eps) -> None:
    """foreach_adamw_step (optimizer.py:80-116) as one native multi-tensor launch."""
    rows, ct, cs = [], [], []
    for ti, (p, g, m, v) in enumerate(zip(params, grads, exp_avgs, exp_avg_sqs)):
        rows.append([p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), 0, p.numel()])
        for s in range(0, p.numel(), _ADAM_CHUNK):
            ct.append(ti)
            cs.append(s)
    if not rows:
        return
    dev = params[0].device
    nv.adamw(_table(rows, dev), torch.tensor(ct, dtype=torch.int32).to(dev), torch.tensor(cs, dtype=torch.int64).to(dev),
             _ADAM_CHUNK, lr, wd, beta1, beta2, eps, step)
