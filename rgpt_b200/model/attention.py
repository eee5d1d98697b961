"""Attention with the reference's submodules (model/attention.py:10-64).

q/k/v/out projections (no bias), QKNorm over d_head, the G1 gate (one Linear(d_head, d_head) shared by
all heads, applied to the normalised q), RoPE and causal attention with dropout on the probabilities.

Inside GPT the engine runs this as: QKV GEMM -> qkv_prep kernel (QK norm, RoPE, gate input) -> gate GEMM
with a bias+sigmoid epilogue -> tcgen05 flash attention with the gate product fused -> out_proj GEMM with
the residual epilogue. Attention.forward on its own (a [B, T, d] CUDA input, as the reference module is
called) runs the same kernels through _AttentionFunction, whose backward is the engine's attention
backward; only the residual add stays outside, as in the reference module.
"""
import torch
import torch.nn as nn

from .. import native as nv
from .norm import QKNorm
from .rope import RotaryEmbedding


class _AttentionFunction(torch.autograd.Function):
    """out = out_proj(gate * causal_attention(rope(qknorm(x Wq^T)), rope(qknorm(x Wk^T)), x Wv^T)).

    Operands are bf16 with fp32 accumulation; the output and the input gradient are fp32. The QK-norm
    parameters (RMSNorm weights or L2Norm temperatures) and the gate are optional inputs."""

    @staticmethod
    def forward(ctx, x, wq, wk, wv, wo, wg, bg, nq, nk, attn, p_drop):
        B, T, d = x.shape
        H, M = attn.n_heads, B * T
        dev, bf = x.device, torch.bfloat16
        spec = attn._qk_spec()
        inv_freq = attn.rotary_emb.inv_freq.float().contiguous()
        xb = x.reshape(M, d).to(bf).contiguous()
        wqkv = torch.cat([wq.detach(), wk.detach(), wv.detach()], 0).to(bf).contiguous()
        qkv = torch.empty(M, 3 * d, device=dev, dtype=bf)
        nv.gemm(xb, wqkv, qkv)
        gated = wg is not None
        qk = torch.empty(M, 2 * d, device=dev, dtype=bf)
        qn = torch.empty(M, d, device=dev, dtype=bf) if gated else None
        nv.qkv_prep_fwd(qkv, qk, qn, inv_freq, spec["kind"], spec["eps"], spec["alpha"], M, T, H, wq=spec["wq"],
                        wk=spec["wk"], sq=spec["sq"], sk=spec["sk"])
        gate = wgb = None
        if gated:
            wgb = wg.detach().to(bf).contiguous()
            gate = torch.empty(M, d, device=dev, dtype=bf)
            nv.gemm(qn.view(M * H, 64), wgb, gate.view(M * H, 64), epi=nv.EPI_BIAS_SIGMOID_BF16,
                    colscale=bg.detach().float().contiguous())
        drop = None
        if p_drop > 0:
            mask = torch.empty(B * H, (T + 31) // 32, T, device=dev, dtype=torch.int32)
            drop = nv.Drop(mask, attn._drop_seed(dev), 2, p_drop)
            nv.attn_drop_mask(drop, B, T, H)
        o = torch.empty(M, d, device=dev, dtype=bf)
        og = torch.empty(M, d, device=dev, dtype=bf) if gated else None
        lse = torch.empty(B, H, T, device=dev, dtype=torch.float32)
        nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H, drop=drop)
        wob = wo.detach().to(bf).contiguous()
        out = torch.empty(M, d, device=dev, dtype=torch.float32)
        nv.gemm(og if gated else o, wob, out, epi=nv.EPI_STORE_F32)
        ctx.save_for_backward(xb, wqkv, qkv, qk, qn, gate, o, og, lse, wob, wgb, inv_freq,
                              drop.mask if drop is not None else None)
        ctx.meta = (B, T, H, d, spec, p_drop, x.dtype, nq is not None, nk is not None)
        return out.view(B, T, d).to(x.dtype)

    @staticmethod
    def backward(ctx, dout):
        xb, wqkv, qkv, qk, qn, gate, o, og, lse, wob, wgb, inv_freq, mask = ctx.saved_tensors
        B, T, H, d, spec, p_drop, xdt, has_nq, has_nk = ctx.meta
        M, dev, bf, f32 = B * T, xb.device, torch.bfloat16, torch.float32
        gated = gate is not None
        drop = nv.Drop(mask, None, 2, p_drop) if mask is not None else None
        dy = dout.reshape(M, d).to(bf).contiguous()
        dog = torch.empty(M, d, device=dev, dtype=bf)
        nv.gemm(dy, wob.t(), dog)                                          # d(og) = dy Wo
        dwo = torch.zeros(d, d, device=dev, dtype=f32)
        nv.gemm(dy.t(), (og if gated else o).t(), dwo, epi=nv.EPI_ACCUM_F32, splitk=0)  # dWo = dy^T og
        do = torch.empty(M, d, device=dev, dtype=bf)
        dgp = torch.empty(M, d, device=dev, dtype=bf) if gated else None
        Dvec = torch.empty(B, H, T, device=dev, dtype=f32)
        dqa = torch.empty(M, d, device=dev, dtype=f32)
        nv.attn_bwd_prep(dog, o, gate, do, dgp, Dvec, B, T, H, dq_zero=dqa)
        dka = torch.empty(M, d, device=dev, dtype=f32)
        dqkv = torch.empty(M, 3 * d, device=dev, dtype=bf)
        nv.attn_bwd(qk, qkv, do, lse, Dvec, dqa, dka, dqkv[:, 2 * d:], B, T, H, drop=drop)
        dqn_gate = dwg = dbg = None
        if gated:
            dgp2 = dgp.view(M * H, 64)
            dqn_gate = torch.empty(M, d, device=dev, dtype=f32)
            nv.gemm(dgp2, wgb.t(), dqn_gate.view(M * H, 64), epi=nv.EPI_STORE_F32)
            dwg = torch.zeros(64, 64, device=dev, dtype=f32)
            nv.gemm(dgp2.t(), qn.view(M * H, 64).t(), dwg, epi=nv.EPI_ACCUM_F32, splitk=0)
            dbg = torch.zeros(64, device=dev, dtype=f32)
        affine, temp = spec["kind"] == nv.NORM_RMS_AFFINE, spec["kind"] == nv.NORM_L2_TEMP
        dnq = torch.zeros_like(spec["wq"], dtype=f32) if has_nq else None
        dnk = torch.zeros_like(spec["wk"], dtype=f32) if has_nk else None
        nv.qkv_prep_bwd(qkv, dqa, dka, dqn_gate, dgp, dqkv, inv_freq, spec["kind"], spec["eps"], spec["alpha"],
                        M, T, H, dbg=dbg, dwq=dnq if affine else None, dwk=dnk if affine else None,
                        dtq=dnq if temp else None, dtk=dnk if temp else None, wq=spec["wq"], wk=spec["wk"],
                        sq=spec["sq"], sk=spec["sk"])
        dwqkv = torch.zeros(3 * d, d, device=dev, dtype=f32)
        nv.gemm(dqkv.t(), xb.t(), dwqkv, epi=nv.EPI_ACCUM_F32, splitk=0)   # dWqkv = dqkv^T x
        dx = torch.empty(M, d, device=dev, dtype=f32)
        nv.gemm(dqkv, wqkv.t(), dx, epi=nv.EPI_STORE_F32)                 # dx = dqkv Wqkv
        return (dx.view(B, T, d).to(xdt), dwqkv[:d], dwqkv[d:2 * d], dwqkv[2 * d:], dwo, dwg, dbg, dnq, dnk,
                None, None)


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
        # plain attributes (not state): what the native kernels need to know about the QK norm
        self.qk_normtype = config.qk_normtype
        self.norm_eps = config.norm_eps
        self._seed = None

    def _qk_spec(self):
        from .engine import qk_norm_spec

        return qk_norm_spec(self, self.qk_normtype, self.norm_eps)

    def _drop_seed(self, dev):
        """Philox key of this module's attention dropout: drawn once from torch's default generator, kept
        on the device and advanced before every dropout forward."""
        if self._seed is None or self._seed.device != dev:
            self._seed = torch.tensor([int(torch.randint(0, 2 ** 62, (1,)))], dtype=torch.int64).to(dev)
        self._seed.add_(1)
        return self._seed

    def forward(self, x):
        """Attention.forward (model/attention.py:35-64) on the native kernels: x [B, T, d_model] CUDA."""
        if not x.is_cuda:
            raise RuntimeError("rgpt_b200 Attention runs on CUDA tensors only (no CPU path)")
        if self.d_head != 64:
            raise ValueError(f"native attention needs head_dim 64, got {self.d_head}")
        spec = self._qk_spec()
        nq = spec["wq"] if spec["wq"] is not None and spec["wq"].requires_grad else None
        nk = spec["wk"] if spec["wk"] is not None and spec["wk"].requires_grad else None
        wg = self.gate_proj.weight if self.g1_gate else None
        bg = self.gate_proj.bias if self.g1_gate else None
        p = float(self.dropout_p) if self.training else 0.0
        return _AttentionFunction.apply(x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                                        self.out_proj.weight, wg, bg, nq, nk, self, p)

