"""Attention with the reference's submodules (model/attention.py:10-64).

q/k/v/out projections (no bias), QKNorm over d_head, the G1 gate (one
Linear(d_head, d_head) shared by all heads, applied to the normalised q), RoPE
and causal attention. Inside GPT this runs as: QKV GEMM -> qkv_prep kernel ->
tcgen05 flash attention with the gate fused -> out_proj GEMM with the residual
epilogue. Attention.forward on its own runs the same kernels through a
one-layer engine (see transformer_block.BlockFunction).
"""
import torch.nn as nn

from .norm import QKNorm
from .rope import RotaryEmbedding


class Attention(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.n_heads = config.n_heads
        self.d_model = config.d_model
        assert self.d_model % self.n_heads == 0, "d_model must be divisible by n_heads"
        self.d_head = self.d_model // self.n_heads
        self.g1_gate = config.g1_gate
        self.q_proj = nn.Linear(self.d_model, self.d_model, bias=False)
        self.k_proj = nn.Linear(self.d_model, self.d_model, bias=False)
        self.v_proj = nn.Linear(self.d_model, self.d_model, bias=False)
        self.out_proj = nn.Linear(self.d_model, self.d_model, bias=False)
        self.qk_norm = (QKNorm(self.d_head, config.qk_normtype, config.norm_eps)
                        if config.qk_normtype != "none" else None)
        if self.g1_gate:
            self.gate_proj = nn.Linear(self.d_head, self.d_head, bias=True)
            nn.init.constant_(self.gate_proj.bias, 1.0)
        self.rotary_emb = RotaryEmbedding(self.d_head, max_seq_len=config.max_seq_len)
        self.dropout_p = config.dropout

    def forward(self, x):
        raise RuntimeError("Attention runs inside GPT's native engine (rgpt_b200.model.GPT)")
