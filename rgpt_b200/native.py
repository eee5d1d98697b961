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

ACTIVATIONS = {"none": 0, "identity": 0, "squared_relu": 1, "gelu": 2, "silu": 3, "mish": 4}


def act_id(name: str) -> int:
    try:
        return ACTIVATIONS[name]
    except KeyError as e:
        raise ValueError(f"unknown activation {name!r}") from e


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


def gemm(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor, *, epi: int = EPI_STORE_BF16,
         act: int = 0, alpha: float = 1.0, beta: float = 0.0, out2: torch.Tensor | None = None,
         c: torch.Tensor | None = None, colscale: torch.Tensor | None = None, splitk: int = 1) -> torch.Tensor:
    """out = epilogue(A @ B^T) for logical A [(b,) M, K] and B [(b,) N, K] (bf16).

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
    _lib.call("rgpt_gemm_bf16",
              ptr(A), a_mn, lda, abs_, ptr(B), b_mn, ldb, bbs,
              M, N, K, batch, epi, act, float(alpha), float(beta),
              d, ldd, dbs, d2, ldd2, d2bs, cp, ldc, cbs,
              ptr(colscale), splitk, _lib.stream_ptr(out.device))
    return out
