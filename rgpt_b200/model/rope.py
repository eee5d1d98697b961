"""RotaryEmbedding with the reference's buffer (model/rope.py:5-57).

Rotation is applied inside the QKV-prep kernel (rotate-half, base 10000,
angles t * inv_freq in fp32); this module keeps the `inv_freq` buffer and the
constructor signature so state_dicts and configs interchange."""
import torch
import torch.nn as nn


class RotaryEmbedding(nn.Module):
    def __init__(self, d_head, max_seq_len=2048, base=10000):
        super().__init__()
        self.d_head = d_head
        self.max_seq_len = max_seq_len
        self.base = base
        inv_freq = 1.0 / (self.base ** (torch.arange(0, self.d_head, 2).float() / self.d_head))
        self.register_buffer("inv_freq", inv_freq)

    def forward(self, q, k):
        raise RuntimeError("RoPE runs fused inside the attention QKV-prep kernel; call Attention or GPT")
