"""TransformerBlock (model/transformer_block.py:10-57): pre-norm attention + FFN residuals with
optional layer scale and branch dropout.

Inside GPT the engine runs the block as fused kernels (the residual add, layer scale and branch dropout
live in the epilogue of each branch's output GEMM). Called on its own, forward(x) composes the native
submodules: the norm kernels, Attention's native forward and the fused linear+activation FFN; the
branch dropout is this module's nn.Dropout, as in the reference."""
import torch
import torch.nn as nn

from .attention import Attention
from .feed_forward import FeedForward
from .norm import functional_l2_norm, functional_rms_norm, get_norm_fn


class TransformerBlock(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.norm_type = config.norm_type
        self.norm_eps = config.norm_eps
        self.use_layer_scale = config.use_layer_scale
        self.attn = Attention(config)
        self.ff = FeedForward(config)
        self.dropout = nn.Dropout(config.dropout)
        if self.norm_type == "f_rmsnorm":
            self.attn_norm = lambda x: functional_rms_norm(x, self.norm_eps)
            self.ff_norm = lambda x: functional_rms_norm(x, self.norm_eps)
        elif self.norm_type == "f_l2norm":
            self.attn_norm = lambda x: functional_l2_norm(x, self.norm_eps)
            self.ff_norm = lambda x: functional_l2_norm(x, self.norm_eps)
        else:
            self.attn_norm = get_norm_fn(config.norm_type, config.d_model, config.norm_eps)
            self.ff_norm = get_norm_fn(config.norm_type, config.d_model, config.norm_eps)
        if self.use_layer_scale:
            self.attn_layer_scale = nn.Parameter(torch.ones(config.d_model))
            self.ff_layer_scale = nn.Parameter(torch.ones(config.d_model))
        if hasattr(self.attn, "out_proj"):
            self.attn.out_proj.RESIDUAL_SCALE_FLAG = True
        if hasattr(self.ff, "out_proj"):
            self.ff.out_proj.RESIDUAL_SCALE_FLAG = True

    def forward(self, x):
        """x [B, T, d] (CUDA) -> h + drop(ff(ff_norm(h))) * ls_ff, h = x + drop(attn(attn_norm(x))) * ls_attn."""
        h = self._residual_branch(x, self.attn_norm, self.attn, "attn_layer_scale")
        return self._residual_branch(h, self.ff_norm, self.ff, "ff_layer_scale")

    def _residual_branch(self, x, norm, sublayer, scale_name):
        branch = self.dropout(sublayer(norm(x)))
        if self.use_layer_scale:
            branch = branch * getattr(self, scale_name)
        return x + branch
