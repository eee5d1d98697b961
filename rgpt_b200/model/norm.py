"""Norm modules with the reference's names, parameters and buffers (model/norm.py).

Inside GPT the native engine fuses these into its kernels (rownorm_fwd/bwd for the residual stream,
qkv_prep for the QK norms). Called on their own, every norm runs the native row-norm kernels through
_RowNormFunction: CUDA tensors, any last dimension (the QK norms' d_head = 64 included), fp32 math,
with the gradients of the input and of the learned weight (RMSNorm) or temperature (L2Norm).
"""
import torch
import torch.nn as nn

from .. import native as nv


class _RowNormFunction(torch.autograd.Function):
    """y = norm(x) over the last dim. `param` is RMSNorm's weight [d], L2Norm's temperature [1] or None;
    the kernels read it on the device."""

    @staticmethod
    def forward(ctx, x, param, kind, eps, alpha):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).float().contiguous()
        p = param.detach().float().contiguous() if param is not None else None
        y = torch.empty_like(x2)
        nv.rownorm_any_fwd(x2, y, kind, eps, w=p, alpha=alpha)
        ctx.save_for_backward(x2, p)
        ctx.meta = (kind, eps, alpha, shape, x.dtype, param.dtype if param is not None else None)
        # the reference's output dtype: x's, promoted with the parameter's (model/norm.py:27-34, :50-51)
        out_dt = torch.promote_types(x.dtype, param.dtype) if param is not None else x.dtype
        return y.view(shape).to(out_dt)

    @staticmethod
    def backward(ctx, gy):
        x2, p = ctx.saved_tensors
        kind, eps, alpha, shape, xdt, pdt = ctx.meta
        dy = gy.reshape(-1, shape[-1]).float().contiguous()
        dx = torch.empty_like(x2)
        dp = torch.zeros_like(p) if p is not None else None
        nv.rownorm_any_bwd(x2, dy, kind, eps, dx, w=p, alpha=alpha,
                           dw=dp if kind == nv.NORM_RMS_AFFINE else None,
                           dtemp=dp if kind == nv.NORM_L2_TEMP else None)
        return dx.view(shape).to(xdt), (dp.to(pdt) if dp is not None else None), None, None, None


def _native_norm(x, kind, eps, param=None, alpha=0.5):
    if not x.is_cuda:
        raise RuntimeError("rgpt_b200 norms run on CUDA tensors only (no CPU path)")
    return _RowNormFunction.apply(x, param, kind, float(eps), float(alpha))


class RMSNorm(nn.Module):
    """Gemma RMSNorm, x * rsqrt(mean(x^2) + eps) * (1 + w) (model/norm.py:8-34)."""

    def __init__(self, dim: int, eps: float = 1e-6, add_unit_offset: bool = True):
        super().__init__()
        self.register_buffer("eps", torch.tensor(float(eps)))
        self.add_unit_offset = add_unit_offset
        self.weight = nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        if not self.add_unit_offset:
            raise NotImplementedError("only the (1 + w) RMSNorm variant is native")
        return _native_norm(x, nv.NORM_RMS_AFFINE, float(self.eps), self.weight)


def functional_rms_norm(x, eps=1e-5):
    """F.rms_norm with its default eps, finfo(x.dtype).eps; `eps` is ignored (model/norm.py:37-38)."""
    return _native_norm(x, nv.NORM_RMS, torch.finfo(x.dtype).eps)


def functional_hyperball_norm(x):
    return _native_norm(x, nv.NORM_HYPERBALL, 0.0)


class L2Norm(nn.Module):
    """x / (||x|| + eps) * temp (model/norm.py:44-51)."""

    def __init__(self, d_model, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.temp = nn.Parameter(torch.ones(1))

    def forward(self, x):
        return _native_norm(x, nv.NORM_L2_TEMP, self.eps, self.temp)


def functional_l2_norm(x, eps=1e-5):
    return _native_norm(x, nv.NORM_L2, eps)


class HybridElasticNorm(nn.Module):
    """Rigid above radius sqrt(d), elastic (s^alpha) below (model/norm.py:58-95)."""

    def __init__(self, dim: int, alpha: float = 0.5, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.alpha = alpha
        self.eps = eps
        self.target_radius = dim ** 0.5

    def forward(self, x):
        return _native_norm(x, nv.NORM_ELASTIC, self.eps, alpha=self.alpha)


class ElasticBallNorm(nn.Module):
    """scale = (sqrt(d) / ||x||)^alpha (model/norm.py:97-132)."""

    def __init__(self, dim: int, alpha: float = 0.5, eps: float = 1e-6):
        super().__init__()
        self.alpha = alpha
        self.eps = eps
        self.target_radius = dim ** 0.5

    def forward(self, x):
        return _native_norm(x, nv.NORM_ELASTICBALL, self.eps, alpha=self.alpha)


class DualElasticBallNorm(nn.Module):
    def __init__(self, dim: int, alpha_q: float = 0.5, alpha_k: float = 0.5, eps: float = 1e-6):
        super().__init__()
        self.q_norm = ElasticBallNorm(dim, alpha=alpha_q, eps=eps)
        self.k_norm = ElasticBallNorm(dim, alpha=alpha_k, eps=eps)

    def forward(self, q, k):
        return self.q_norm(q), self.k_norm(k)


class AsymmetricHyperballNorm(nn.Module):
    def __init__(self, dim, scale_q=1.0, scale_k=1.1):
        super().__init__()
        self.register_buffer("scale_q", torch.tensor(scale_q))
        self.register_buffer("scale_k", torch.tensor(scale_k))

    def forward(self, q, k):
        return functional_hyperball_norm(q) * self.scale_q, functional_hyperball_norm(k) * self.scale_k


class HyperballNorm(nn.Module):
    def forward(self, x):
        return functional_hyperball_norm(x)


def get_norm_fn(name, d_model, eps):
    """Norm module by config name (model/norm.py:165-179)."""
    if name == "rmsnorm":
        return RMSNorm(d_model, eps)
    if name == "layernorm":
        return nn.LayerNorm(d_model, eps)
    if name == "l2norm":
        return L2Norm(d_model, eps)
    if name == "elastic":
        return HybridElasticNorm(d_model, eps=eps)
    if name == "elasticball":
        return ElasticBallNorm(d_model, eps=eps)
    if name == "hyperball":
        return HyperballNorm()
    return nn.Identity()


class QKNorm(nn.Module):
    """Per-head q/k normalisation (model/norm.py:182-204). Runs fused in the QKV-prep kernel."""

    def __init__(self, d_head, norm_type, norm_eps, alpha_q: float = 0.5, alpha_k: float = 0.5,
                 scale_q: float = 1.0, scale_k: float = 1.1):
        super().__init__()
        self.norm_type = norm_type
        if norm_type == "f_rmsnorm":
            self.q_norm_fn = lambda q: functional_rms_norm(q, norm_eps)
            self.k_norm_fn = lambda k: functional_rms_norm(k, norm_eps)
        elif norm_type == "f_l2norm":
            self.q_norm_fn = lambda q: functional_l2_norm(q, norm_eps)
            self.k_norm_fn = lambda k: functional_l2_norm(k, norm_eps)
        elif norm_type == "dual_elasticball":
            self.norm_module = DualElasticBallNorm(d_head, alpha_q=alpha_q, alpha_k=alpha_k, eps=norm_eps)
        elif norm_type == "asymmetric_hyperball":
            self.norm_module = AsymmetricHyperballNorm(d_head, scale_q=scale_q, scale_k=scale_k)
        else:
            self.q_norm_fn = get_norm_fn(norm_type, d_head, norm_eps)
            self.k_norm_fn = get_norm_fn(norm_type, d_head, norm_eps)

    def forward(self, q, k):
        """Normalise q and k over d_head (model/norm.py:200-204) with the native row-norm kernels. Inside
        Attention and GPT the same norm runs fused in the QKV-prep kernel instead."""
        if hasattr(self, "norm_module"):
            return self.norm_module(q, k)
        return self.q_norm_fn(q), self.k_norm_fn(k)
