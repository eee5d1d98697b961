"""FusedLinearActivationFunction: act(x @ W1^T) @ W2 on tcgen05 GEMMs (model/kernels.py:289-374).

Forward: one GEMM with the activation epilogue writes pre and post (bf16), a
second GEMM computes post @ W2. Backward: dW2 = post^T dY; dpre = (dY W2^T) *
act'(pre) in the GEMM epilogue; dW1 = dpre^T x; dX = dpre W1. Operands are
bf16 with fp32 accumulation; transposed operands are read MN-major in place.
"""
import torch

from .. import native as nv


class FusedLinearActivationFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W1, W2, activation="squared_relu"):
        if not x.is_cuda:
            raise RuntimeError("FusedLinearActivationFunction runs on CUDA tensors only (no CPU path)")
        act = nv.act_id(activation)
        M, K = x.shape
        N = W1.shape[0]
        Out = W2.shape[1]
        xb = x.contiguous().to(torch.bfloat16)
        w1b = W1.contiguous().to(torch.bfloat16)
        w2b = W2.to(torch.bfloat16)  # [N, Out]; any strides with one unit stride
        if w2b.stride(0) != 1 and w2b.stride(1) != 1:
            w2b = w2b.contiguous()
        pre = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        post = torch.empty_like(pre)
        nv.gemm(xb, w1b, pre, epi=nv.EPI_ACT_FWD, act=act, out2=post)
        out = torch.empty(M, Out, device=x.device, dtype=torch.bfloat16)
        nv.gemm(post, w2b.t(), out)
        ctx.save_for_backward(xb, w1b, w2b, pre, post)
        ctx.act = act
        ctx.dtypes = (x.dtype, W1.dtype, W2.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        xb, w1b, w2b, pre, post = ctx.saved_tensors
        dy = grad_output.contiguous().to(torch.bfloat16)
        M, K = xb.shape
        N, Out = w2b.shape
        dW2 = torch.zeros(N, Out, device=dy.device, dtype=torch.float32)
        nv.gemm(post.t(), dy.t(), dW2, epi=nv.EPI_ACCUM_F32, splitk=0)
        dpre = torch.empty(M, N, device=dy.device, dtype=torch.bfloat16)
        nv.gemm(dy, w2b, dpre, epi=nv.EPI_ACT_BWD, act=ctx.act, c=pre)
        dW1 = torch.zeros(N, K, device=dy.device, dtype=torch.float32)
        nv.gemm(dpre.t(), xb.t(), dW1, epi=nv.EPI_ACCUM_F32, splitk=0)
        dx = torch.empty(M, K, device=dy.device, dtype=torch.float32)
        nv.gemm(dpre, w1b.t(), dx, epi=nv.EPI_STORE_F32)
        xd, w1d, w2d = ctx.dtypes
        return dx.to(xd), dW1.to(w1d), dW2.to(w2d), None
