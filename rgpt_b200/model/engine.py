"""Native execution engine for GPT / rGPT (forward, fused loss, backward).

The engine replaces the reference's eager/autograd execution of
model/gpt.py:92-143, model/transformer_block.py:43-57, model/attention.py:35-64,
model/feed_forward.py:25-37 and trainer.py:139-167 with one hand-scheduled
sequence of sm_100a kernels per micro-batch:

  forward  (per layer application)        backward (reverse order)
  ------------------------------------    ------------------------------------------
  rownorm_fwd  x -> hn (bf16)             ACT_BWD GEMM   dpre = (df W2) * act'(pre)
  GEMM         qkv = hn Wqkv^T            ACCUM GEMMs    dW2 += df^T post, dW1 += dpre^T hn2
  qkv_prep     QK-norm, gate, RoPE        GEMM           dhn2 = dpre W1 (fp32)
  attn_fwd     o, og = o*gate, lse        rownorm_bwd    g += norm'(h) dhn2, da = bf16(g*ls_attn)
  RESID GEMM   h = x + (og Wo^T) ls       GEMM/ACCUM     dog = da Wo, dWo += da^T og
  rownorm_fwd  h -> hn2                   attn_bwd_prep, attn_bwd, qkv_prep_bwd -> dqkv
  ACT_FWD GEMM pre, post                  ACCUM GEMM     dWqkv += dqkv^T hn; GEMM dhn = dqkv Wqkv
  RESID GEMM   x' = h + (post W2^T) ls    rownorm_bwd    g += norm'(x) dhn, df_prev = bf16(g*ls_ff)

Parameters stay fp32 nn.Parameters with the reference's names; the engine keeps
bf16 "shadow" copies for the GEMM operands (refreshed when a parameter's
version changes, and written directly by the optimizer kernels), and owns one
flat fp32 gradient arena whose views are attached as every parameter's .grad.
Weight gradients are ACCUMULATED into the arena by the GEMM epilogues, so
gradient accumulation and shared (recurrent) layers need no extra adds.
"""
from __future__ import annotations

import math

from typing import Dict, List

import torch

from .. import native as nv

NORM_KINDS = {
    "rmsnorm": nv.NORM_RMS_AFFINE,
    "f_rmsnorm": nv.NORM_RMS,
    "l2norm": nv.NORM_L2_TEMP,
    "f_l2norm": nv.NORM_L2,
    "elastic": nv.NORM_ELASTIC,
    "elasticball": nv.NORM_ELASTICBALL,
    "dual_elasticball": nv.NORM_ELASTICBALL,
    "hyperball": nv.NORM_HYPERBALL,
    "asymmetric_hyperball": nv.NORM_HYPERBALL,
}


def norm_spec(kind_name: str, module, eps: float, is_qk: bool = False):
    """(kind, eps, alpha, weight, temp_param) for a norm by config name.

    f_rmsnorm uses F.rms_norm's default eps = finfo(float32).eps (model/norm.py:37-38)."""
    if kind_name in ("identity", "none", None) or kind_name not in NORM_KINDS:
        if kind_name == "layernorm":
            raise NotImplementedError("layernorm residual norms are not on the native path")
        return nv.NORM_IDENTITY, 0.0, 0.5, None, None
    kind = NORM_KINDS[kind_name]
    if kind == nv.NORM_RMS:
        return kind, nv.FLT_EPS, 0.5, None, None
    temp = getattr(module, "temp", None) if kind == nv.NORM_L2_TEMP else None
    # RMSNorm's weight, or L2Norm's learned temperature: the kernels read either from the device, so a
    # captured step sees the optimizer's latest value and nothing waits for a host copy
    w = getattr(module, "weight", None) if kind == nv.NORM_RMS_AFFINE else temp
    e = float(getattr(module, "eps", eps)) if module is not None and not torch.is_tensor(
        getattr(module, "eps", None)) else float(eps)
    return kind, e, 0.5, w, temp


def qk_norm_spec(attn, qk: str, norm_eps: float) -> dict:
    """Arguments of the QKV-prep kernels for an Attention module's QK norm (QKNorm, model/norm.py:182-204):
    kind, eps, alpha, wq/wk (RMSNorm weights, or L2Norm temperatures read on the device), tq/tk (unused
    by-value temperatures) and the constant post-scales sq/sk (asymmetric hyperball)."""
    if qk in ("none", "identity", None) or attn.qk_norm is None:
        return dict(kind=nv.NORM_IDENTITY, eps=0.0, alpha=0.5, wq=None, wk=None, tq=1.0, tk=1.0, sq=1.0, sk=1.0)
    qn = attn.qk_norm
    if qk == "f_rmsnorm":
        return dict(kind=nv.NORM_RMS, eps=nv.FLT_EPS, alpha=0.5, wq=None, wk=None, tq=1.0, tk=1.0, sq=1.0, sk=1.0)
    if qk == "dual_elasticball":
        nm = qn.norm_module
        return dict(kind=nv.NORM_ELASTICBALL, eps=nm.q_norm.eps, alpha=nm.q_norm.alpha, wq=None, wk=None,
                    tq=1.0, tk=1.0, sq=1.0, sk=1.0)
    if qk == "asymmetric_hyperball":
        nm = qn.norm_module
        return dict(kind=nv.NORM_HYPERBALL, eps=0.0, alpha=0.5, wq=None, wk=None, tq=1.0, tk=1.0,
                    sq=float(nm.scale_q), sk=float(nm.scale_k))
    kind, e, alpha, _, _ = norm_spec(qk, qn.q_norm_fn, norm_eps)
    spec = dict(kind=kind, eps=e, alpha=alpha, wq=None, wk=None, tq=1.0, tk=1.0, sq=1.0, sk=1.0)
    if kind == nv.NORM_ELASTIC or kind == nv.NORM_ELASTICBALL:
        spec["eps"] = float(qn.q_norm_fn.eps)
        spec["alpha"] = float(qn.q_norm_fn.alpha)
    if kind == nv.NORM_RMS_AFFINE:
        spec["eps"] = float(qn.q_norm_fn.eps)
        spec["wq"], spec["wk"] = qn.q_norm_fn.weight, qn.k_norm_fn.weight
    if kind == nv.NORM_L2_TEMP:
        spec["eps"] = float(qn.q_norm_fn.eps)
        spec["wq"], spec["wk"] = qn.q_norm_fn.temp, qn.k_norm_fn.temp  # read on the device
    return spec


class _Acts:
    """Activation buffers for one (B, T) shape, reused across steps."""

    def __init__(self, eng, B, T, dev):
        c = eng.cfg
        d, V, F = c["d_model"], c["vocab_size"], 4 * c["d_model"]
        H = c["n_heads"]
        M = B * T
        self.B, self.T, self.M = B, T, M
        napp = eng.n_apps
        e = lambda *s, dt=torch.bfloat16: torch.empty(*s, device=dev, dtype=dt)
        f32 = torch.float32
        self.x = [e(M, d, dt=f32) for _ in range(napp + 1)]
        self.hn = [e(M, d) for _ in range(napp)]
        self.qkv = [e(M, 3 * d) for _ in range(napp)]
        self.qk = [e(M, 2 * d) for _ in range(napp)]
        self.gate = [e(M, d) for _ in range(napp)] if eng.g1 else [None] * napp
        self.qn = [e(M, d) for _ in range(napp)] if eng.g1 else [None] * napp
        self.o = [e(M, d) for _ in range(napp)]
        self.og = [e(M, d) for _ in range(napp)] if eng.g1 else self.o
        self.lse = [e(B, H, T, dt=f32) for _ in range(napp)]
        self.h = [e(M, d, dt=f32) for _ in range(napp)]
        self.hn2 = [e(M, d) for _ in range(napp)]
        # squared ReLU keeps only the post-activation (its derivative is 2 sqrt(post)); the others the pre too
        self.pre = [e(M, F) for _ in range(napp)] if eng.act != nv.ACT_SQRELU else [None] * napp
        self.post = [e(M, F) for _ in range(napp)]
        self.a_raw = [e(M, d, dt=f32) for _ in range(napp)] if eng.ls else [None] * napp
        self.f_raw = [e(M, d, dt=f32) for _ in range(napp)] if eng.ls else [None] * napp
        self.hf = e(M, d)
        self.logits = e(M, V)
        R = eng.n_recur if eng.halting else 0
        if R:
            self.hq = e(R, M, d)
            self.q = e(R, M, 2, dt=f32)
            self.dq = e(R, M, 2, dt=f32)
            self.argmax = e(R, M, dt=torch.int32)
            # per-column-tile partial maxima of the per-recurrence lm_head (its logits are never stored)
            self.amax_val = e(M, (V + 127) // 128, dt=f32)
            self.amax_idx = e(M, (V + 127) // 128, dt=torch.int32)
        # backward scratch
        self.g = e(M, d, dt=f32)
        self.gb = e(M, d)
        self.dy32 = e(M, d, dt=f32)
        self.dpre = e(M, F)
        self.dog = e(M, d)
        self.do = e(M, d)
        self.dgp = e(M, d)
        self.D = e(B, H, T, dt=f32)
        self.dqa = e(M, d, dt=f32)
        self.dka = e(M, d, dt=f32)
        self.dqkv = e(M, 3 * d)
        # loss scalars: [total, token, halt, q_cont], CE scale buffer, per-row losses
        self.losses = torch.zeros(4, device=dev, dtype=f32)
        self.scale_buf = torch.zeros(2, device=dev, dtype=f32)
        self.loss_rows = e(M, dt=f32)
        # dropout keep bits, written by the forward and read by the backward (p > 0 only):
        # embedding / residual branches [M, d/32], attention probabilities [B*H, ceil(T/32), T]
        if eng.p_drop > 0:
            i32 = torch.int32
            self.drop_emb = e(M, d // 32, dt=i32)
            self.drop_a = [e(M, d // 32, dt=i32) for _ in range(napp)]
            self.drop_f = [e(M, d // 32, dt=i32) for _ in range(napp)]
            self.drop_att = [e(B * H, (T + 31) // 32, T, dt=i32) for _ in range(napp)]


class Engine:
    def __init__(self, model):
        self.model = model
        c = model.config
        self.cfg = c
        self.d = c["d_model"]
        self.H = c["n_heads"]
        if self.d != self.H * 64:
            raise ValueError(f"native attention needs head_dim 64 (d_model={self.d}, n_heads={self.H})")
        self.L = c["n_layers"]
        self.n_recur = c.get("n_recur", 1)
        self.n_apps = self.L * self.n_recur
        self.halting = bool(c.get("cal_halt_loss", False)) and self.n_recur > 1
        self.detach_recur = bool(c.get("detach_recur", False))
        self.ls = bool(c.get("use_layer_scale", False))
        self.g1 = bool(c.get("g1_gate", False))
        self.act = nv.act_id(c["activation_type"])
        self.V = c["vocab_size"]
        self.ignore_index = c.get("pad_token_id", -100)
        if self.ignore_index is None:
            self.ignore_index = -100
        self.device = model.lm_head.weight.device
        if self.device.type != "cuda":
            raise RuntimeError("the native engine runs on CUDA devices only (no CPU path)")
        self.p_drop = float(c.get("dropout", 0.0) or 0.0)
        if not 0.0 <= self.p_drop < 1.0:
            raise ValueError(f"dropout must be in [0, 1), got {self.p_drop}")
        if self.p_drop > 0 and self.d % 128 != 0:
            raise ValueError("native dropout needs d_model % 128 == 0")
        # Philox key of the dropout masks: drawn from torch's default generator (so torch.manual_seed
        # makes runs repeatable), kept on the device and advanced by one before every dropout forward,
        # inside a captured step too.
        seed = int(torch.randint(0, 2 ** 62, (1,), dtype=torch.int64))
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            # data-parallel ranks seeded alike still draw independent masks
            seed ^= (torch.distributed.get_rank() * 0x9E3779B97F4A7C15) & (2 ** 62 - 1)
        self.drop_seed = torch.tensor([seed], dtype=torch.int64).to(self.device)
        self._drop_active = False
        self._rng_stream = None
        self._mask_events = []
        self.overlap_masks = True  # draw the dropout masks on a side stream (False: on the caller's)
        self._build_param_views()
        self._acts = {}
        self._spec_cache = {}

    # ------------------------------------------------------------------ parameters
    def _build_param_views(self):
        m = self.model
        dev = self.device
        named = list(m.named_parameters())
        # every gradient starts on a 16-byte boundary (the GEMM epilogues' TMA and vector stores need
        # it), so 1-element parameters such as L2Norm's temperature are padded to 4 floats
        slot = lambda n: (n + 3) // 4 * 4  # noqa: E731
        total = sum(slot(p.numel()) for _, p in named)
        self.grad_arena = torch.zeros(total, device=dev, dtype=torch.float32)
        off = 0
        self.grads = {}
        # gradient buckets, in the order the backward finishes them: the parameters after the
        # layers (ln_f, lm_head, ...), each layer from the last to the first, then the embedding
        spans: Dict[str, List[int]] = {}
        for name, p in named:
            g = self.grad_arena[off:off + p.numel()].view_as(p)
            p.grad = g
            p._rgpt_grad_arena = self.grad_arena
            self.grads[name] = g
            parts = name.split(".")
            key = f"layer{parts[1]}" if parts[0] == "layers" else ("pre" if not any(k.startswith("layer") for k in spans)
                                                                       else "post")
            sp = spans.setdefault(key, [off, off])
            if sp[1] != off:
                raise RuntimeError(f"gradient bucket {key} is not contiguous in the arena")
            sp[1] = off + slot(p.numel())
            off += slot(p.numel())
        self.grad_buckets = spans
        # bf16 shadows: fused QKV per layer, out, fc1, fc2, lm_head
        d = self.d
        self.shadow_src = []  # (param, shadow view, version)
        self.layer_w = []
        for blk in m.layers:
            at, ff = blk.attn, blk.ff
            wqkv = torch.empty(3 * d, d, device=dev, dtype=torch.bfloat16)
            views = {"q": wqkv[0:d], "k": wqkv[d:2 * d], "v": wqkv[2 * d:3 * d]}
            for key, lin in (("q", at.q_proj), ("k", at.k_proj), ("v", at.v_proj)):
                self._add_shadow(lin.weight, views[key])
            wo = torch.empty(d, d, device=dev, dtype=torch.bfloat16)
            w1 = torch.empty(4 * d, d, device=dev, dtype=torch.bfloat16)
            w2 = torch.empty(d, 4 * d, device=dev, dtype=torch.bfloat16)
            self._add_shadow(at.out_proj.weight, wo)
            self._add_shadow(ff.fc1.weight, w1)
            self._add_shadow(ff.fc2.weight, w2)
            wg = None
            if self.g1:
                wg = torch.empty(64, 64, device=dev, dtype=torch.bfloat16)
                self._add_shadow(at.gate_proj.weight, wg)
            gq = self.grads_of(at.q_proj.weight)
            dwqkv = torch.as_strided(self.grad_arena, (3 * d, d), (d, 1), gq.storage_offset())
            # q, k, v are registered consecutively, so their arena slices form one [3d, d] block
            assert dwqkv[2 * d:].data_ptr() == self.grads_of(at.v_proj.weight).data_ptr()
            self.layer_w.append(dict(wqkv=wqkv, wo=wo, w1=w1, w2=w2, wg=wg, dwqkv=dwqkv))
        self.lm_w = torch.empty(self.V, d, device=dev, dtype=torch.bfloat16)
        self._add_shadow(m.lm_head.weight, self.lm_w)
        rope = m.layers[0].attn.rotary_emb
        self.inv_freq = rope.inv_freq.detach().to(dev, torch.float32).contiguous()

    def grads_of(self, p):
        return p.grad

    def _add_shadow(self, p, view):
        p._rgpt_shadow = view
        self.shadow_src.append([p, view, None])

    def sync_shadows(self):
        """Refresh bf16 shadows whose fp32 parameter changed outside the optimizer kernels."""
        for ent in self.shadow_src:
            p, view, ver = ent
            if ver != p._version:
                with torch.no_grad():
                    view.copy_(p.detach())
                ent[2] = p._version

    def mark_shadows_fresh(self):
        for ent in self.shadow_src:
            ent[2] = ent[0]._version

    def zero_grad(self):
        self.grad_arena.zero_()

    def acts(self, B, T):
        key = (B, T)
        if key not in self._acts:
            self._acts.clear()  # one live shape at a time keeps HBM use bounded
            self._acts[key] = _Acts(self, B, T, self.device)
        return self._acts[key]

    # ------------------------------------------------------------------ helpers
    def _norm(self, module_or_none, kind_name):
        return norm_spec(kind_name, module_or_none, self.cfg["norm_eps"])

    def _qk_spec(self, attn):
        spec = self._spec_cache.get(("qk", id(attn)))
        if spec is None:
            spec = self._qk_spec_uncached(attn)
            self._spec_cache[("qk", id(attn))] = spec
        return spec

    def _qk_spec_uncached(self, attn):
        return qk_norm_spec(attn, self.cfg.get("qk_normtype", "f_rmsnorm"), self.cfg["norm_eps"])

    def _resid_norm(self, blk_or_model, which):
        """(kind, eps, alpha, w, temp) for the residual-stream norm `which` of a block / the model."""
        key = ("res", id(blk_or_model), which)
        spec = self._spec_cache.get(key)
        if spec is None:
            spec = self._resid_norm_uncached(blk_or_model, which)
            self._spec_cache[key] = spec
        return spec

    def _resid_norm_uncached(self, blk_or_model, which):
        nt = self.cfg["norm_type"]
        mod = getattr(blk_or_model, which)
        mod = mod if isinstance(mod, torch.nn.Module) else None
        kind, eps, alpha, w, temp = norm_spec(nt, mod, self.cfg["norm_eps"])
        if mod is not None and hasattr(mod, "eps"):
            ev = mod.eps
            eps = float(ev.item() if torch.is_tensor(ev) else ev) if kind != nv.NORM_RMS else eps
        if mod is not None and hasattr(mod, "alpha"):
            alpha = float(mod.alpha)
        return kind, eps, alpha, w, temp

    # ------------------------------------------------------------------ forward
    @torch.no_grad()
    def forward(self, input_ids, labels=None, *, training=True, want_loss=False, grad_scale=1.0):
        """Run the model forward (and, with want_loss, the fused loss + in-place dlogits).

        Returns the _Acts holding logits / losses. grad_scale multiplies the stored dlogits."""
        m = self.model
        self.sync_shadows()
        B, T = input_ids.shape
        A = self.acts(B, T)
        M, d, H = A.M, self.d, self.H
        ids = input_ids.reshape(-1)
        if ids.dtype != torch.int64:
            ids = ids.long()
        self._ids = ids.contiguous()
        lab = None
        if labels is not None:
            lab = labels.reshape(-1)
            lab = (lab if lab.dtype == torch.int64 else lab.long()).contiguous()
        self._labels = lab
        # nn.Dropout is active in training mode (model/gpt.py:96, transformer_block.py:45,52, attention.py:57)
        self._drop_active = m.training and self.p_drop > 0
        if self._drop_active:
            self.drop_seed.add_(1)
            self._draw_masks(A)
        nv.embedding_fwd(self._ids, m.embs.weight, A.x[0], drop=self._drop(A, "emb"))
        halting = self.halting and lab is not None
        self._halting_active = halting
        app = 0
        for r in range(self.n_recur):
            for li, blk in enumerate(m.layers):
                self._layer_fwd(blk, self.layer_w[li], A, app)
                app += 1
            if halting:
                kind, eps, alpha, w, temp = self._resid_norm(m, "ln_f")
                nv.rownorm_fwd(A.x[app], A.hq[r], kind, eps, w=w, temp=1.0,
                               alpha=alpha, qw=m.q_head.weight, qb=m.q_head.bias, qout=A.q[r])
                # per-step logits feed only the no-grad argmax (their CE is discarded, model/gpt.py:113-117):
                # the lm_head GEMM reduces each row to its argmax in the epilogue instead of storing them
                nv.gemm_argmax(A.hq[r], self.lm_w, A.amax_val, A.amax_idx, A.argmax[r])
        kind, eps, alpha, w, temp = self._resid_norm(m, "ln_f")
        nv.rownorm_fwd(A.x[app], A.hf, kind, eps, w=w, temp=1.0, alpha=alpha)
        nv.gemm(A.hf, self.lm_w, A.logits)
        if want_loss:
            A.losses.zero_()
            nv.cross_entropy(A.logits, lab, ignore_index=self.ignore_index, grad_scale=grad_scale,
                             loss_rows=A.loss_rows, scale_buf=A.scale_buf, loss_out=A.losses[1:2],
                             write_grad=training)
            if halting:
                nv.halt_losses(A.q, A.argmax, lab, A.dq, A.losses[2:4], grad_scale=grad_scale)
            torch.sum(A.losses[1:4], dim=0, keepdim=True, out=A.losses[0:1])
        return A

    # dropout sites: the embedding, and per layer application app: 4*app + 0 (attention branch),
    # + 1 (FFN branch), + 2 (attention probabilities)
    EMB_DROP_SITE = 0xFFFFFF

    def _drop(self, A, kind, app=0):
        """The Drop spec of one site, or None when dropout is off for this pass."""
        if not self._drop_active:
            return None
        if kind == "emb":
            return nv.Drop(A.drop_emb, self.drop_seed, self.EMB_DROP_SITE, self.p_drop)
        if kind == "attn_out":
            return nv.Drop(A.drop_a[app], self.drop_seed, 4 * app, self.p_drop)
        if kind == "ff_out":
            return nv.Drop(A.drop_f[app], self.drop_seed, 4 * app + 1, self.p_drop)
        return nv.Drop(A.drop_att[app], self.drop_seed, 4 * app + 2, self.p_drop)

    def _draw_masks(self, A):
        """Draw every layer application's dropout masks (attention probabilities and both residual
        branches) on a side stream that forks here, after the seed increment; each layer's attention
        waits for its own masks (events), so the Philox work overlaps the layers before it and the
        QKV projection and preparation of its own layer."""
        main = torch.cuda.current_stream()
        if self.overlap_masks:
            if self._rng_stream is None:
                self._rng_stream = torch.cuda.Stream(device=self.device)
            st = self._rng_stream
            st.wait_stream(main)
        else:
            st = main  # in stream order, e.g. to time the other kernels without overlap
        if len(self._mask_events) < self.n_apps:
            self._mask_events = [torch.cuda.Event() for _ in range(self.n_apps)]
        with torch.cuda.stream(st):
            for app in range(self.n_apps):
                nv.attn_drop_mask(self._drop(A, "attn_p", app), A.B, A.T, self.H)
                nv.drop_mask_rows(self._drop(A, "attn_out", app), A.M, self.d)
                nv.drop_mask_rows(self._drop(A, "ff_out", app), A.M, self.d)
                self._mask_events[app].record(st)

    def _layer_fwd(self, blk, W, A, app):
        d, H, B, T, M = self.d, self.H, A.B, A.T, A.M
        at = blk.attn
        x = A.x[app]
        kind, eps, alpha, w, temp = self._resid_norm(blk, "attn_norm")
        nv.rownorm_fwd(x, A.hn[app], kind, eps, w=w, temp=1.0, alpha=alpha)
        nv.gemm(A.hn[app], W["wqkv"], A.qkv[app])
        qs = self._qk_spec(at)
        nv.qkv_prep_fwd(A.qkv[app], A.qk[app], A.qn[app], self.inv_freq, qs["kind"], qs["eps"], qs["alpha"],
                        M, T, H, wq=qs["wq"], wk=qs["wk"], tq=qs["tq"], tk=qs["tk"], sq=qs["sq"], sk=qs["sk"])
        if self.g1:
            # G1 gate = sigmoid(q_n Wg^T + bg), one [M*H, 64] x [64, 64] GEMM with a bias+sigmoid epilogue
            nv.gemm(A.qn[app].view(M * H, 64), W["wg"], A.gate[app].view(M * H, 64),
                    epi=nv.EPI_BIAS_SIGMOID_BF16, colscale=at.gate_proj.bias)
        if self._drop_active:
            torch.cuda.current_stream().wait_event(self._mask_events[app])
        nv.attn_fwd(A.qk[app], A.qkv[app], A.gate[app], A.o[app], A.og[app] if self.g1 else None, A.lse[app],
                    B, T, H, drop=self._drop(A, "attn_p", app))
        nv.gemm(A.og[app], W["wo"], A.h[app], epi=nv.EPI_RESID_F32, c=x,
                colscale=blk.attn_layer_scale if self.ls else None, out2=A.a_raw[app],
                drop=self._drop(A, "attn_out", app))
        kind, eps, alpha, w, temp = self._resid_norm(blk, "ff_norm")
        nv.rownorm_fwd(A.h[app], A.hn2[app], kind, eps, w=w, temp=1.0,
                       alpha=alpha)
        if self.act == nv.ACT_SQRELU:  # post = relu(h W1^T)^2 only (no pre-activation written)
            nv.gemm(A.hn2[app], W["w1"], A.post[app], epi=nv.EPI_ACT_FWD, act=nv.ACT_SQRELU_POST)
        else:
            nv.gemm(A.hn2[app], W["w1"], A.pre[app], epi=nv.EPI_ACT_FWD, act=self.act, out2=A.post[app])
        nv.gemm(A.post[app], W["w2"], A.x[app + 1], epi=nv.EPI_RESID_F32, c=A.h[app],
                colscale=blk.ff_layer_scale if self.ls else None, out2=A.f_raw[app],
                drop=self._drop(A, "ff_out", app))

    # ------------------------------------------------------------------ backward
    @torch.no_grad()
    def backward(self, A, dlogits=None, alpha_dev=None):
        """Backpropagate from dlogits (bf16 [M, V]; default: the in-place dlogits of the fused loss).

        alpha_dev: optional device scalar scaling every gradient (the upstream loss gradient)."""
        m = self.model
        G = self.grads
        dl = A.logits if dlogits is None else dlogits
        # lm_head: dhf = dl W_lm ; dW_lm += dl^T hf
        nv.gemm(dl, self.lm_w.t(), A.dy32, epi=nv.EPI_STORE_F32, alpha_dev=alpha_dev)
        nv.gemm(dl.t(), A.hf.t(), G["lm_head.weight"], epi=nv.EPI_ACCUM_F32, splitk=0, alpha_dev=alpha_dev)
        napp = self.n_apps
        last_blk = m.layers[(napp - 1) % self.L]
        kind, eps, alpha, w, temp = self._resid_norm(m, "ln_f")
        lnf_w = "ln_f.weight" if kind == nv.NORM_RMS_AFFINE else None
        lnf_t = "ln_f.temp" if kind == nv.NORM_L2_TEMP else None
        tval = 1.0
        halting = self._halting_active
        need_gb_now = not halting
        # A data-parallel optimizer may hook the arena to reduce each gradient bucket as soon as the
        # backward has finished it (overlapping the collective with the rest of the backward). Buckets
        # are final after one pass only without recurrence reuse or halting heads.
        sync = getattr(self.grad_arena, "_rgpt_sync", None)
        if sync is not None and (self.n_recur != 1 or halting):
            sync = None
        if sync is not None:
            sync.begin(self.grad_arena)
        nv.rownorm_bwd(A.x[napp], A.dy32, kind, eps, A.g, w=w, temp=tval, alpha=alpha, g_in=None,
                       g_bf16=A.gb if need_gb_now else None,
                       ls=last_blk.ff_layer_scale if (self.ls and need_gb_now) else None,
                       raw=A.f_raw[napp - 1] if need_gb_now else None,
                       dls=G[self._pname(last_blk, "ff_layer_scale")] if (self.ls and need_gb_now) else None,
                       dw=G[lnf_w] if lnf_w else None, dtemp=G[lnf_t] if lnf_t else None,
                       drop=self._drop(A, "ff_out", napp - 1) if need_gb_now else None)
        if halting:
            if alpha_dev is not None:
                A.dq.mul_(alpha_dev)
        if sync is not None and "post" in self.grad_buckets:
            sync.ready(self.grad_arena, *self.grad_buckets["post"])
        app = napp
        for r in reversed(range(self.n_recur)):
            if halting:
                # q-head gradient at the end of recurrence r joins g before that recurrence's layers
                blk = m.layers[self.L - 1]
                nv.rownorm_bwd(A.x[app], None, kind, eps, A.g, w=w, temp=tval, alpha=alpha, g_in=A.g,
                               g_bf16=A.gb, ls=blk.ff_layer_scale if self.ls else None,
                               raw=A.f_raw[app - 1], dls=G[self._pname(blk, "ff_layer_scale")] if self.ls else None,
                               dw=G[lnf_w] if lnf_w else None, dtemp=G[lnf_t] if lnf_t else None,
                               dq=A.dq[r], qw=m.q_head.weight, h=A.hq[r], dqw=G["q_head.weight"],
                               dqb=G["q_head.bias"], drop=self._drop(A, "ff_out", app - 1))
            for li in reversed(range(self.L)):
                app -= 1
                first = app == 0
                boundary = li == 0 and r > 0
                # at a detached recurrence boundary only the q-head gradient flows into the previous step
                cut = self.detach_recur and boundary
                # with halting, the q-head pass at the boundary emits bf16(g*ls) and the layer-scale grad
                # from the complete gradient, so the layer must not emit them first
                defer = halting and boundary
                self._layer_bwd(m.layers[li], li, self.layer_w[li], A, app, first or cut or defer)
                if sync is not None:
                    sync.ready(self.grad_arena, *self.grad_buckets[f"layer{li}"])
                if cut:
                    A.g.zero_()
                    A.gb.zero_()
        nv.embedding_bwd(self._ids, A.g, G["embs.weight"], drop=self._drop(A, "emb"))
        if sync is not None:
            if "pre" in self.grad_buckets:
                sync.ready(self.grad_arena, *self.grad_buckets["pre"])
            sync.end(self.grad_arena)

    def _pname(self, blk, attr):
        idx = list(self.model.layers).index(blk)
        return f"layers.{idx}.{attr}"

    def _layer_bwd(self, blk, li, W, A, app, first):
        """Backward of one layer application. On entry A.g = dL/dx_out (fp32) and A.gb = bf16(g * ls_ff)."""
        G = self.grads
        d, H, B, T, M = self.d, self.H, A.B, A.T, A.M
        pre = f"layers.{li}."
        # ---------------- FFN
        if self.act == nv.ACT_SQRELU:  # act'(pre) = 2 sqrt(post)
            nv.gemm(A.gb, W["w2"].t(), A.dpre, epi=nv.EPI_ACT_BWD, act=nv.ACT_SQRELU_POST, c=A.post[app])
        else:
            nv.gemm(A.gb, W["w2"].t(), A.dpre, epi=nv.EPI_ACT_BWD, act=self.act, c=A.pre[app])
        nv.gemm(A.gb.t(), A.post[app].t(), G[pre + "ff.fc2.weight"], epi=nv.EPI_ACCUM_F32, splitk=0)
        nv.gemm(A.dpre, W["w1"].t(), A.dy32, epi=nv.EPI_STORE_F32)
        nv.gemm(A.dpre.t(), A.hn2[app].t(), G[pre + "ff.fc1.weight"], epi=nv.EPI_ACCUM_F32, splitk=0)
        kind, eps, alpha, w, temp = self._resid_norm(blk, "ff_norm")
        nv.rownorm_bwd(A.h[app], A.dy32, kind, eps, A.g, w=w, temp=1.0,
                       alpha=alpha, g_in=A.g, g_bf16=A.gb, ls=blk.attn_layer_scale if self.ls else None,
                       raw=A.a_raw[app], dls=G[pre + "attn_layer_scale"] if self.ls else None,
                       dw=G[pre + "ff_norm.weight"] if kind == nv.NORM_RMS_AFFINE else None,
                       dtemp=G[pre + "ff_norm.temp"] if kind == nv.NORM_L2_TEMP else None,
                       drop=self._drop(A, "attn_out", app))
        # ---------------- attention
        at = blk.attn
        nv.gemm(A.gb, W["wo"].t(), A.dog)
        nv.gemm(A.gb.t(), A.og[app].t(), G[pre + "attn.out_proj.weight"], epi=nv.EPI_ACCUM_F32, splitk=0)
        nv.attn_bwd_prep(A.dog, A.o[app], A.gate[app], A.do, A.dgp if self.g1 else None, A.D, B, T, H,
                         dq_zero=A.dqa)
        nv.attn_bwd(A.qk[app], A.qkv[app], A.do, A.lse[app], A.D, A.dqa, A.dka, A.dqkv[:, 2 * d:], B, T, H,
                    drop=self._drop(A, "attn_p", app))
        qs = self._qk_spec(at)
        qn = pre + "attn.qk_norm."
        dqn_gate = None
        if self.g1:
            # gate backward on tensor cores: d q_n += dgp Wg ; dWg += dgp^T q_n (split-K over M*H rows)
            dgp2 = A.dgp.view(M * H, 64)
            dqn_gate = A.dy32.view(M * H, 64)
            nv.gemm(dgp2, W["wg"].t(), dqn_gate, epi=nv.EPI_STORE_F32)
            nv.gemm(dgp2.t(), A.qn[app].view(M * H, 64).t(), G[pre + "attn.gate_proj.weight"],
                    epi=nv.EPI_ACCUM_F32, splitk=0)
        nv.qkv_prep_bwd(A.qkv[app], A.dqa, A.dka, dqn_gate, A.dgp if self.g1 else None, A.dqkv,
                        self.inv_freq, qs["kind"], qs["eps"], qs["alpha"], M, T, H,
                        dbg=G[pre + "attn.gate_proj.bias"] if self.g1 else None,
                        dwq=G.get(qn + "q_norm_fn.weight"), dwk=G.get(qn + "k_norm_fn.weight"),
                        dtq=G.get(qn + "q_norm_fn.temp"), dtk=G.get(qn + "k_norm_fn.temp"),
                        wq=qs["wq"], wk=qs["wk"], tq=qs["tq"], tk=qs["tk"], sq=qs["sq"], sk=qs["sk"])
        nv.gemm(A.dqkv.t(), A.hn[app].t(), W["dwqkv"], epi=nv.EPI_ACCUM_F32, splitk=0)
        nv.gemm(A.dqkv, W["wqkv"].t(), A.dy32, epi=nv.EPI_STORE_F32)
        kind, eps, alpha, w, temp = self._resid_norm(blk, "attn_norm")
        prev_blk = None if first else self.model.layers[(app - 1) % self.L]
        nv.rownorm_bwd(A.x[app], A.dy32, kind, eps, A.g, w=w, temp=1.0,
                       alpha=alpha, g_in=A.g,
                       g_bf16=None if first else A.gb,
                       ls=prev_blk.ff_layer_scale if (self.ls and prev_blk is not None) else None,
                       raw=None if first else A.f_raw[app - 1],
                       dls=G[self._pname(prev_blk, "ff_layer_scale")] if (self.ls and prev_blk is not None) else None,
                       dw=G[pre + "attn_norm.weight"] if kind == nv.NORM_RMS_AFFINE else None,
                       dtemp=G[pre + "attn_norm.temp"] if kind == nv.NORM_L2_TEMP else None,
                       drop=None if first else self._drop(A, "ff_out", app - 1))
