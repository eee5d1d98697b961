"""RotaryEmbedding with the reference's buffer and constructor (model/rope.py:5-57).

Inside Attention and GPT the rotation runs fused in the QKV-prep kernel. Called on its own,
forward(q, k) rotates [B, H, T, d_head] CUDA tensors with the native rgpt_rope kernel: rotate-half RoPE,
angles t * inv_freq[j] and their cos/sin in fp32 for every input dtype (the reference builds its
cos/sin cache in q's dtype, which for fp32 inputs is the same arithmetic), output in the input's dtype.
"""
import torch
import torch.nn as nn

from .. import native as nv


def _rotate(t: torch.Tensor, inv_freq: torch.Tensor, backward: bool) -> torch.Tensor:
    src = t if t.dtype == torch.float32 and t.stride(-1) == 1 else t.float().contiguous()
    out = torch.empty(src.shape, device=src.device, dtype=torch.float32)
    nv.rope(src, out, inv_freq, backward=backward)
    return out if t.dtype == torch.float32 else out.to(t.dtype)


class _RopeFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, inv_freq):
        ctx.save_for_backward(inv_freq)
        return _rotate(q, inv_freq, False), _rotate(k, inv_freq, False)

    @staticmethod
    def backward(ctx, gq, gk):
        (inv_freq,) = ctx.saved_tensors
        dq = _rotate(gq, inv_freq, True) if gq is not None else None
        dk = _rotate(gk, inv_freq, True) if gk is not None else None
        return dq, dk, None


class RotaryEmbedding(nn.Module):
    def __init__(self, d_head, max_seq_len=2048, base=10000):
        super().__init__()
        self.d_head = d_head
        self.max_seq_len = max_seq_len
        self.base = base
        inv_freq = 1.0 / (self.base ** (torch.arange(0, self.d_head, 2).float() / self.d_head))
        self.register_buffer("inv_freq", inv_freq)

    def forward(self, q, k):
        """q, k: [batch, heads, seq, d_head] CUDA tensors -> (q, k) rotated (model/rope.py:38-51)."""
        if not (q.is_cuda and k.is_cuda):
            raise RuntimeError("rgpt_b200 RotaryEmbedding runs on CUDA tensors only (no CPU path)")
        if q.dim() != 4 or k.dim() != 4 or q.shape[-1] != self.d_head or k.shape[-1] != self.d_head:
            raise ValueError(f"q and k must be [batch, heads, seq, {self.d_head}]")
        inv_freq = self.inv_freq.to(q.device, torch.float32).contiguous()
        return _RopeFunction.apply(q, k, inv_freq)
