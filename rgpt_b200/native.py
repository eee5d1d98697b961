"""Torch-tensor wrappers over the C ABI (include/rgpt.h).

Each function validates shapes/dtypes on the host, then enqueues one or more
native kernels on the current CUDA stream. None of them has a fallback.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_ACCUM_F32 = 2
EPI_ACT_FWD = 3
EPI_ACT_BWD = 4
EPI_RESID_F32 = 5
EPI_POLY_BF16 = 6
EPI_BIAS_SIGMOID_BF16 = 7
EPI_POLY_F32 = 8
EPI_ARGMAX_BF16 = 9

ACTIVATIONS = {"none": 0, "identity": 0, "squared_relu": 1, "gelu": 2, "silu": 3, "mish": 4}
ACT_SQRELU = 1
ACT_SQRELU_POST = 5  # squared ReLU with the post-activation as the only forward output and the backward's C


def act_id(name: str) -> int:
    try:
        return ACTIVATIONS[name]
    except KeyError as e:
        raise ValueError(f"unknown activation {name!r}") from e


class Drop:
    """Dropout of one site: keep bits are drawn from Philox4x32-10 under the device seed (int64 [1])
    and the site number, and stored in `mask` (int32 words) for the backward; p is the drop rate."""

    __slots__ = ("mask", "seed", "site", "p")

    def __init__(self, mask: torch.Tensor, seed: torch.Tensor | None, site: int, p: float):
        if mask.dtype != torch.int32 or not mask.is_contiguous():
            raise ValueError("dropout masks are contiguous int32 words")
        if seed is not None and (seed.dtype != torch.int64 or seed.numel() != 1):
            raise ValueError("dropout seed is a device int64 [1]")
        if not 0.0 <= p < 1.0:
            raise ValueError(f"dropout p must be in [0, 1), got {p}")
        self.mask, self.seed, self.site, self.p = mask, seed, int(site), float(p)


def _drop_args(drop: "Drop | None", seed_needed: bool = True):
    if drop is None:
        return None, None, 0, 0.0
    if seed_needed and drop.seed is None:
        raise ValueError("this dropout call draws new bits and needs the seed")
    return ptr(drop.mask), ptr(drop.seed) if drop.seed is not None else None, drop.site & 0xFFFFFFFF, drop.p


def gemm_argmax(A: torch.Tensor, B: torch.Tensor, part_val: torch.Tensor, part_idx: torch.Tensor,
                argmax: torch.Tensor) -> None:
    """argmax[m] = first index of the maximum of bf16(A @ B^T)[m, :] without writing the product.

    A [M, K], B [N, K] bf16 with unit stride on K; part_val (fp32) / part_idx (int32) [M, >= ceil(N/128)]
    hold the per-column-tile partial results; argmax int32 [M]."""
    M, K = A.shape
    N = B.shape[0]
    for t, n in ((A, "A"), (B, "B")):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.dim() != 2:
            raise ValueError(f"gemm_argmax: {n} must be 2-D bf16 with unit stride on K")
    if part_val.dtype != torch.float32 or part_idx.dtype != torch.int32 or argmax.dtype != torch.int32:
        raise TypeError("gemm_argmax: partial values fp32, partial indices and argmax int32")
    ld = part_val.stride(0)
    if part_idx.stride(0) != ld or part_val.shape[0] < M or part_val.shape[1] < (N + 127) // 128:
        raise ValueError("gemm_argmax: partial buffers must be [M, >= ceil(N/128)] with equal row strides")
    _lib.call("rgpt_gemm_argmax", ptr(A), A.stride(0), ptr(B), B.stride(0), M, N, K, ptr(part_val), ptr(part_idx),
              ld, ptr(argmax), _lib.stream_ptr(A.device))


def drop_mask_rows(drop: Drop, M: int, N: int) -> None:
    """Fill drop.mask [M, ceil(N/32)] with the residual-branch keep bits of (seed, site)."""
    if drop.mask.dim() != 2 or drop.mask.shape[0] < M:
        raise ValueError("row dropout mask must be [M, ceil(N/32)] words")
    dm, ds, dsite, dp = _drop_args(drop)
    _lib.call("rgpt_drop_mask", dm, drop.mask.stride(0), ds, dsite, dp, M, N, _lib.stream_ptr(drop.mask.device))


def attn_drop_mask(drop: Drop, B: int, T: int, H: int) -> None:
    """Fill drop.mask [B*H, ceil(T/32), T] with the attention-probability keep bits of (seed, site)."""
    if drop.mask.numel() < B * H * ((T + 31) // 32) * T:
        raise ValueError("attention dropout mask must hold [B*H, ceil(T/32), T] words")
    dm, ds, dsite, dp = _drop_args(drop)
    _lib.call("rgpt_attn_drop_mask", dm, ds, dsite, dp, B, T, H, _lib.stream_ptr(drop.mask.device))


def _operand(t: torch.Tensor):
    """(mn_major, ld, bstride) for a logical [.., rows, K] bf16 operand view."""
    if t.dtype != torch.bfloat16:
        raise TypeError(f"GEMM operands must be bf16, got {t.dtype}")
    if t.stride(-1) == 1:
        mn, ld = 0, t.stride(-2)
    elif t.stride(-2) == 1:
        mn, ld = 1, t.stride(-1)
    else:
        raise ValueError(f"GEMM operand needs a unit stride in one of its last two dims, got {t.stride()}")
    bstride = t.stride(0) if t.dim() == 3 else 0
    return mn, ld, bstride


def _out(t: torch.Tensor | None):
    if t is None:
        return None, 0, 0
    if t.stride(-1) != 1:
        raise ValueError("GEMM outputs/epilogue inputs must have unit column stride")
    return ptr(t), t.stride(-2), (t.stride(0) if t.dim() == 3 else 0)


# Optional GEMM timing hook: when set to a list, every gemm() call appends
# (start_event, end_event, flops, (epi, M, N, K, batch)) recorded on the launching stream.
gemm_events: list | None = None


def gemm(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor, *, epi: int = EPI_STORE_BF16,
         act: int = 0, alpha: float = 1.0, beta: float = 0.0, out2: torch.Tensor | None = None,
         c: torch.Tensor | None = None, colscale: torch.Tensor | None = None, splitk: int = 1,
         alpha_dev: torch.Tensor | None = None, drop: Drop | None = None) -> torch.Tensor:
    """out = epilogue(A @ B^T) for logical A [(b,) M, K] and B [(b,) N, K] (bf16).

    drop (RESID_F32 only): branch dropout whose mask drop_mask_rows filled.

    Either operand may be K-major (unit stride on K) or MN-major (unit stride
    on M/N), e.g. ``gemm(dy.t(), x.t(), dw, epi=EPI_ACCUM_F32)`` computes
    dW += dy^T x without materialising a transpose.
    """
    if A.dim() != B.dim() or A.dim() not in (2, 3):
        raise ValueError("A and B must both be 2-D or both 3-D")
    M, K = A.shape[-2], A.shape[-1]
    N, K2 = B.shape[-2], B.shape[-1]
    if K != K2:
        raise ValueError(f"inner dims differ: {K} vs {K2}")
    batch = A.shape[0] if A.dim() == 3 else 1
    if out.shape[-2:] != (M, N):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected [..., {M}, {N}]")
    a_mn, lda, abs_ = _operand(A)
    b_mn, ldb, bbs = _operand(B)
    d, ldd, dbs = _out(out)
    d2, ldd2, d2bs = _out(out2)
    cp, ldc, cbs = _out(c)
    ev = gemm_events
    if ev is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
    if drop is None:
        _lib.call("rgpt_gemm_bf16",
                  ptr(A), a_mn, lda, abs_, ptr(B), b_mn, ldb, bbs,
                  M, N, K, batch, epi, act, float(alpha), float(beta),
                  d, ldd, dbs, d2, ldd2, d2bs, cp, ldc, cbs,
                  ptr(colscale), splitk, ptr(alpha_dev), _lib.stream_ptr(out.device))
    else:
        dm, _, _, dp = _drop_args(drop, seed_needed=False)
        _lib.call("rgpt_gemm_bf16_dropout",
                  ptr(A), a_mn, lda, abs_, ptr(B), b_mn, ldb, bbs,
                  M, N, K, batch, epi, act, float(alpha), float(beta),
                  d, ldd, dbs, d2, ldd2, d2bs, cp, ldc, cbs,
                  ptr(colscale), splitk, ptr(alpha_dev), dm, drop.mask.shape[-1], dp,
                  _lib.stream_ptr(out.device))
    if ev is not None:
        e1.record()
        ev.append((e0, e1, 2.0 * M * N * K * batch, (epi, M, N, K, batch)))
    return out


# ----------------------------------------------------------------------------- attention
def _check(t, dtype, name):
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit column stride")


def attn_fwd(qk: torch.Tensor, qkv: torch.Tensor, gate: torch.Tensor | None, o: torch.Tensor,
             og: torch.Tensor | None, lse: torch.Tensor, B: int, T: int, H: int, drop: Drop | None = None) -> None:
    """Causal attention over token-major q/k (qk [B*T, 2d]) and v (qkv[:, 2d:3d]).

    Writes o [B*T, d] (bf16), og = o * gate (if gate given) and lse [B, H, T] (fp32).
    drop: attention-probability dropout; its mask must have been filled by attn_drop_mask."""
    d = H * 64
    for t, n in ((qk, "qk"), (qkv, "qkv"), (o, "o")):
        _check(t, torch.bfloat16, n)
    if qk.shape != (B * T, 2 * d) or qkv.shape != (B * T, 3 * d) or o.shape != (B * T, d):
        raise ValueError("attention shapes do not match [B*T, 2d] / [B*T, 3d] / [B*T, d]")
    if lse.dtype != torch.float32 or lse.numel() != B * H * T:
        raise ValueError("lse must be fp32 [B, H, T]")
    if drop is not None and drop.mask.numel() < B * H * ((T + 31) // 32) * T:
        raise ValueError("attention dropout mask must hold [B*H, ceil(T/32), T] words")
    dm, _, _, dp = _drop_args(drop, seed_needed=False)
    _lib.call("rgpt_attn_fwd", ptr(qk), ptr(qkv), ptr(gate), ptr(o), ptr(og), ptr(lse), B, T, H, d,
              dm, dp, _lib.stream_ptr(o.device))


def attn_bwd_prep(dog: torch.Tensor, o: torch.Tensor, gate: torch.Tensor | None, do: torch.Tensor,
                  dgate_pre: torch.Tensor | None, D: torch.Tensor, B: int, T: int, H: int,
                  dq_zero: torch.Tensor | None = None) -> None:
    """do = dog*gate, dgate_pre = dog*o*gate*(1-gate), D = rowsum(do*o) per (token, head);
    dq_zero (the fp32 [B*T, d] dq accumulator of attn_bwd), when given, is zeroed in the same pass."""
    d = H * 64
    if dq_zero is not None and (dq_zero.dtype != torch.float32 or not dq_zero.is_contiguous()
                                or dq_zero.numel() != B * T * d):
        raise RuntimeError("attn_bwd_prep: dq_zero must be a contiguous fp32 [B*T, d] tensor")
    _lib.call("rgpt_attn_bwd_prep", ptr(dog), ptr(o), ptr(gate), ptr(do), ptr(dgate_pre), ptr(D), ptr(dq_zero),
              B, T, H, d, _lib.stream_ptr(o.device))


def attn_bwd(qk: torch.Tensor, qkv: torch.Tensor, do: torch.Tensor, lse: torch.Tensor, D: torch.Tensor,
             dq: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, B: int, T: int, H: int,
             drop: Drop | None = None) -> None:
    """dq (fp32, accumulated: caller zeroes), dk (fp32) and dv (bf16, may be a strided column view).

    drop: the forward's attention dropout (its mask is read back; no new bits are drawn)."""
    d = H * 64
    if dq.dtype != torch.float32 or dk.dtype != torch.float32 or dv.dtype != torch.bfloat16:
        raise TypeError("dq/dk must be fp32 and dv bf16")
    if drop is not None and drop.mask.numel() < B * H * ((T + 31) // 32) * T:
        raise ValueError("attention dropout mask must hold [B*H, ceil(T/32), T] words")
    dm, _, _, dp = _drop_args(drop, seed_needed=False)
    _lib.call("rgpt_attn_bwd", ptr(qk), ptr(qkv), ptr(do), ptr(lse), ptr(D), ptr(dq), ptr(dk), dk.stride(0),
              ptr(dv), dv.stride(0), B, T, H, d, dm, dp, _lib.stream_ptr(do.device))


# ----------------------------------------------------------------------------- norms
NORM_IDENTITY, NORM_RMS_AFFINE, NORM_RMS, NORM_L2_TEMP, NORM_L2, NORM_ELASTIC, NORM_ELASTICBALL, NORM_HYPERBALL = range(8)
FLT_EPS = 1.1920928955078125e-07  # torch.finfo(torch.float32).eps


def rownorm_fwd(x: torch.Tensor, y: torch.Tensor, kind: int, eps: float, *, w: torch.Tensor | None = None,
                temp: float = 1.0, alpha: float = 0.5, stat: torch.Tensor | None = None,
                qw: torch.Tensor | None = None, qb: torch.Tensor | None = None,
                qout: torch.Tensor | None = None) -> None:
    M, d = x.shape
    _lib.call("rgpt_rownorm_fwd", ptr(x), ptr(y), ptr(stat), ptr(w), float(temp), kind, float(eps), float(alpha),
              M, d, ptr(qw), ptr(qb), ptr(qout), _lib.stream_ptr(x.device))


def rownorm_bwd(x: torch.Tensor, dy: torch.Tensor | None, kind: int, eps: float, g_out: torch.Tensor, *,
                w: torch.Tensor | None = None, temp: float = 1.0, alpha: float = 0.5,
                g_in: torch.Tensor | None = None, g_bf16: torch.Tensor | None = None,
                ls: torch.Tensor | None = None, raw: torch.Tensor | None = None, dls: torch.Tensor | None = None,
                dw: torch.Tensor | None = None, dtemp: torch.Tensor | None = None,
                dq: torch.Tensor | None = None, qw: torch.Tensor | None = None, h: torch.Tensor | None = None,
                dqw: torch.Tensor | None = None, dqb: torch.Tensor | None = None, drop: Drop | None = None) -> None:
    """drop: the dropout of the branch whose gradient g_bf16 is (its mask, read back; no new bits)."""
    M, d = x.shape
    if drop is not None and drop.mask.numel() < M * (d // 32):
        raise ValueError("branch dropout mask must hold [M, d/32] words")
    dm, _, _, dp = _drop_args(drop, seed_needed=False)
    _lib.call("rgpt_rownorm_bwd", ptr(x), ptr(dy), ptr(w), float(temp), kind, float(eps), float(alpha), M, d,
              ptr(g_in), ptr(g_out), ptr(g_bf16), ptr(ls), ptr(raw), ptr(dls), ptr(dw), ptr(dtemp),
              ptr(dq), ptr(qw), ptr(h), ptr(dqw), ptr(dqb), dm, dp, _lib.stream_ptr(x.device))


# ----------------------------------------------------------------------------- standalone modules
def _rows_f32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.float32 or t.dim() != 2 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous fp32 [M, d] tensor")


def rownorm_any_fwd(x: torch.Tensor, y: torch.Tensor, kind: int, eps: float, *, w: torch.Tensor | None = None,
                    alpha: float = 0.5) -> None:
    """y = norm(x) over rows of any length (fp32 [M, d] both); w: RMSNorm weight [d] or L2Norm temp [1]."""
    _rows_f32(x, "x")
    _rows_f32(y, "y")
    if y.shape != x.shape:
        raise ValueError("rownorm_any_fwd: y must have x's shape")
    M, d = x.shape
    _lib.call("rgpt_rownorm_any_fwd", ptr(x), ptr(y), ptr(w), kind, float(eps), float(alpha), M, d,
              _lib.stream_ptr(x.device))


def rownorm_any_bwd(x: torch.Tensor, dy: torch.Tensor, kind: int, eps: float, dx: torch.Tensor, *,
                    w: torch.Tensor | None = None, alpha: float = 0.5, dw: torch.Tensor | None = None,
                    dtemp: torch.Tensor | None = None) -> None:
    """dx = norm'(x)^T dy (written); dw (RMSNorm weight) and dtemp (L2Norm temp) are accumulated."""
    for t, n in ((x, "x"), (dy, "dy"), (dx, "dx")):
        _rows_f32(t, n)
    M, d = x.shape
    _lib.call("rgpt_rownorm_any_bwd", ptr(x), ptr(dy), ptr(w), kind, float(eps), float(alpha), M, d, ptr(dx),
              ptr(dw), ptr(dtemp), _lib.stream_ptr(x.device))


def rope(inp: torch.Tensor, out: torch.Tensor, inv_freq: torch.Tensor, backward: bool = False) -> None:
    """out (contiguous fp32 [B, H, T, D]) = RoPE(inp) for fp32 inp [B, H, T, D] with unit stride on D."""
    if inp.dtype != torch.float32 or inp.dim() != 4 or inp.stride(-1) != 1:
        raise ValueError("rope input must be a 4-D fp32 [B, H, T, D] tensor with unit stride on D")
    if out.dtype != torch.float32 or out.shape != inp.shape or not out.is_contiguous():
        raise ValueError("rope output must be a contiguous fp32 tensor of the input's shape")
    B, H, T, D = inp.shape
    if inv_freq.dtype != torch.float32 or inv_freq.numel() != D // 2 or not inv_freq.is_contiguous():
        raise ValueError("inv_freq must be a contiguous fp32 [D/2] tensor")
    sb, sh, st, _ = inp.stride()
    _lib.call("rgpt_rope", ptr(inp), sb, sh, st, ptr(out), ptr(inv_freq), B, H, T, D, int(backward),
              _lib.stream_ptr(inp.device))


# ----------------------------------------------------------------------------- QKV prep
def qkv_prep_fwd(qkv, qk, qn, inv_freq, qk_kind, eps, alpha, M, T, H, *, wq=None, wk=None,
                 tq=1.0, tk=1.0, sq=1.0, sk=1.0) -> None:
    _lib.call("rgpt_qkv_prep_fwd", ptr(qkv), ptr(qk), ptr(qn), ptr(inv_freq), qk_kind, float(eps), float(alpha),
              ptr(wq), ptr(wk), float(tq), float(tk), float(sq), float(sk), M, T, H, _lib.stream_ptr(qkv.device))


def qkv_prep_bwd(qkv, dq, dk, dqn_gate, dgp, dqkv, inv_freq, qk_kind, eps, alpha, M, T, H, *, dbg=None,
                 dwq=None, dwk=None, dtq=None, dtk=None, wq=None, wk=None, tq=1.0, tk=1.0, sq=1.0, sk=1.0) -> None:
    _lib.call("rgpt_qkv_prep_bwd", ptr(qkv), ptr(dq), ptr(dk), ptr(dqn_gate), ptr(dgp), ptr(dqkv), ptr(dbg),
              ptr(dwq), ptr(dwk), ptr(dtq), ptr(dtk), ptr(inv_freq), qk_kind, float(eps), float(alpha), ptr(wq),
              ptr(wk), float(tq), float(tk), float(sq), float(sk), M, T, H, _lib.stream_ptr(qkv.device))


# ----------------------------------------------------------------------------- embedding / loss
def embedding_fwd(ids: torch.Tensor, emb: torch.Tensor, x: torch.Tensor, drop: Drop | None = None) -> None:
    M = ids.numel()
    V, d = emb.shape
    if drop is not None and drop.mask.numel() < M * (d // 32):
        raise ValueError("embedding dropout mask must hold [M, d/32] words")
    _lib.call("rgpt_embedding_fwd", ptr(ids), ptr(emb), ptr(x), M, d, V, *_drop_args(drop), _lib.stream_ptr(x.device))


def embedding_bwd(ids: torch.Tensor, dx: torch.Tensor, demb: torch.Tensor, drop: Drop | None = None) -> None:
    M = ids.numel()
    V, d = demb.shape
    if drop is not None and drop.mask.numel() < M * (d // 32):
        raise ValueError("embedding dropout mask must hold [M, d/32] words")
    dm, _, _, dp = _drop_args(drop, seed_needed=False)
    _lib.call("rgpt_embedding_bwd", ptr(ids), ptr(dx), ptr(demb), M, d, V, dm, dp, _lib.stream_ptr(dx.device))


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor, *, ignore_index: int = -100, grad_scale: float = 1.0,
                  loss_rows: torch.Tensor | None = None, argmax: torch.Tensor | None = None,
                  scale_buf: torch.Tensor | None = None, loss_out: torch.Tensor | None = None,
                  write_grad: bool = False) -> None:
    M, V = logits.shape
    nk = 1 + (scale_buf is not None) + (loss_out is not None and loss_rows is not None)
    _lib.call("rgpt_cross_entropy", ptr(logits), logits.stride(0), M, V, ptr(labels), int(ignore_index),
              float(grad_scale), ptr(loss_rows), ptr(argmax), ptr(scale_buf), ptr(loss_out), int(write_grad),
              _lib.stream_ptr(logits.device), kernels=nk)


def halt_losses(q: torch.Tensor, argmax: torch.Tensor, labels: torch.Tensor, dq: torch.Tensor,
                losses: torch.Tensor, grad_scale: float = 1.0) -> None:
    R, M = q.shape[0], q.shape[1]
    _lib.call("rgpt_halt_losses", ptr(q), ptr(argmax), ptr(labels), R, M, float(grad_scale), ptr(dq), ptr(losses),
              _lib.stream_ptr(q.device))


# ----------------------------------------------------------------------------- optimizer
# hp: optional device pointer (int) to a parameter group's block of RGPT_HP_FLOATS scalars; when
# given, the kernels read this step's lr / betas / bias corrections from it instead of the arguments.
HP_FLOATS = 8


def adamw(table: torch.Tensor, chunk_tensor: torch.Tensor, chunk_start: torch.Tensor, chunk_elems: int,
          lr: float, wd: float, beta1: float, beta2: float, eps: float, step: int, hp: int | None = None) -> None:
    _lib.call("rgpt_adamw", ptr(table), ptr(chunk_tensor), ptr(chunk_start), chunk_tensor.numel(), chunk_elems,
              float(lr), float(wd), float(beta1), float(beta2), float(eps), int(step), hp,
              _lib.stream_ptr(table.device))


def muon_prep(table, n, R, C, X, beta, nesterov, sumsq, hp: int | None = None) -> None:
    _lib.call("rgpt_muon_prep", ptr(table), n, R, C, ptr(X), X.stride(0), X.stride(1), float(beta), int(nesterov),
              ptr(sumsq), hp, _lib.stream_ptr(X.device))


def ns_scale(X, rows, cols, n, sumsq) -> None:
    _lib.call("rgpt_ns_scale", ptr(X), X.stride(0), X.stride(1), rows, cols, n, ptr(sumsq), _lib.stream_ptr(X.device))


def _ns_src(src: torch.Tensor):
    """(is_bf16, batch/row/col element strides) of a 3-D [n, rows, cols] source view."""
    if src.dim() != 3 or src.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("Newton-Schulz source must be a 3-D fp32/bf16 [n, rows, cols] view")
    return int(src.dtype == torch.bfloat16), src.stride(0), src.stride(1), src.stride(2)


def ns_sumsq(src: torch.Tensor, sumsq: torch.Tensor) -> None:
    """sumsq[b] += ||src[b]||_F^2 (fp32 accumulation)."""
    bf, sb, si, sj = _ns_src(src)
    n, rows, cols = src.shape
    _lib.call("rgpt_ns_sumsq", ptr(src), bf, sb, si, sj, rows, cols, n, ptr(sumsq), _lib.stream_ptr(src.device))


def ns_split(src: torch.Tensor, *, sumsq: torch.Tensor | None = None, xout: torch.Tensor | None = None,
             dst: torch.Tensor | None = None, nblk: int = 0, blk_off: int = 0, lo_mask: int = 0) -> None:
    """v = src / max(||src||_F, 1e-7) (if sumsq given) -> xout (fp32) and nblk bf16 hi/lo blocks of dst.

    Block k starts blk_off elements after dst's first element and holds bf16(v - bf16(v)) if bit k of
    lo_mask is set, else bf16(v). dst and xout share src's [n, rows, cols] indexing (their own strides)."""
    bf, sb, si, sj = _ns_src(src)
    n, rows, cols = src.shape
    if xout is not None and (xout.dtype != torch.float32 or xout.stride(2) != 1):
        raise ValueError("ns_split: xout must be fp32 with unit column stride")
    if dst is not None and (dst.dtype != torch.bfloat16 or dst.stride(2) != 1):
        raise ValueError("ns_split: dst must be bf16 with unit column stride")
    _lib.call("rgpt_ns_split", ptr(src), bf, sb, si, sj, rows, cols, n, ptr(sumsq),
              ptr(xout), xout.stride(0) if xout is not None else 0, xout.stride(1) if xout is not None else 0,
              ptr(dst), dst.stride(0) if dst is not None else 0, dst.stride(1) if dst is not None else 0,
              nblk, blk_off, lo_mask, _lib.stream_ptr(src.device))


def muon_apply(table, n, R, C, X, lr, wd, muon_lr, scale, hp: int | None = None) -> None:
    _lib.call("rgpt_muon_apply", ptr(table), n, R, C, ptr(X), X.stride(0), X.stride(1), float(lr), float(wd),
              float(muon_lr), float(scale), hp, _lib.stream_ptr(X.device))


# ----------------------------------------------------------------------------- data-parallel staging
SEG_CHUNK = 16384


def segment_table(segs, device):
    """Device table and work list of rgpt_segment_copy for segments (tensor, bf16 copy or None, buffer
    offset, element offset in the tensor, count): (table int64 [n, 4], chunk_seg int32, chunk_start int64)."""
    rows, cs, cst = [], [], []
    for i, (t, t2, off, lo, n) in enumerate(segs):
        if not t.is_contiguous() or (t2 is not None and (not t2.is_contiguous() or t2.dtype != torch.bfloat16)):
            raise ValueError("segment tensors must be contiguous (second tensors bf16)")
        rows.append([t.data_ptr() + lo * t.element_size(), t2.data_ptr() + lo * 2 if t2 is not None else 0, off, n])
        for st in range(0, n, SEG_CHUNK):
            cs.append(i)
            cst.append(st)
    if not rows:
        return None
    return (torch.tensor(rows, dtype=torch.int64).to(device), torch.tensor(cs, dtype=torch.int32).to(device),
            torch.tensor(cst, dtype=torch.int64).to(device))


def segment_copy(plan, buf: torch.Tensor, tensor_bf16: bool, scale: float = 1.0, unpack: bool = False) -> None:
    """Pack the plan's segments into buf (unpack=False) or write buf back into them (unpack=True)."""
    if plan is None:
        return
    table, cs, cst = plan
    if buf.dtype not in (torch.float32, torch.bfloat16) or not buf.is_contiguous():
        raise ValueError("staging buffers are contiguous fp32 or bf16")
    _lib.call("rgpt_segment_copy", ptr(table), ptr(cs), ptr(cst), cs.numel(), SEG_CHUNK, ptr(buf),
              int(buf.dtype == torch.bfloat16), int(tensor_bf16), float(scale), int(unpack), _lib.stream_ptr(buf.device))


def ns_chain(X: torch.Tensor, X2: torch.Tensor, A: torch.Tensor, B: torch.Tensor, xr: int, xc: int, steps: int,
             a: float, b: float, c: float, counters: torch.Tensor) -> None:
    """The whole quintic Newton-Schulz iteration of the n matrices X[:, :xr, :xc] (normalised, bf16) in one
    persistent launch; the result lands in X2 for odd `steps`, else in X. A, B [n, >=xr, >=xr] scratch,
    counters int32 [>= n * 3 * steps] (zeroed by the call)."""
    for t, nme in ((X, "X"), (X2, "X2"), (A, "A"), (B, "B")):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.stride(2) != 1:
            raise ValueError(f"ns_chain: {nme} must be a 3-D bf16 tensor with unit column stride")
    if X2.stride() != X.stride() or B.stride() != A.stride():
        raise ValueError("ns_chain: X/X2 and A/B must share strides")
    n = X.shape[0]
    if counters.dtype != torch.int32 or counters.numel() < n * 3 * steps:
        raise ValueError("ns_chain: counters must be int32 with >= n * 3 * steps entries")
    _lib.call("rgpt_ns_chain", ptr(X), ptr(X2), ptr(A), ptr(B), n, xr, xc, X.stride(1), X.stride(0), A.stride(1),
              A.stride(0), int(steps), float(a), float(b), float(c), ptr(counters), _lib.stream_ptr(X.device))
