"""GPT / rGPT with the reference's constructor, parameter names and init (model/gpt.py:11-143).

Two execution paths share one native engine (model/engine.py):

* ``forward(input_ids, labels=None)`` keeps the reference's return value
  ``(final_logits, accum_halt_loss, all_step_q, target_q_continues)`` and is
  differentiable through autograd, so reference-style training code (compute
  the loss on the logits, call backward) works unchanged. Logits are bf16.
* ``forward_loss(input_ids, labels)`` is the training fast path used by the
  Trainer and the benchmark: forward, cross entropy (+ rGPT halting losses)
  and the in-place bf16 dlogits in one pass, then ``loss.backward()`` runs the
  native backward. Returns (total_loss, token_loss, q_loss) as 0-d tensors.

Weight gradients are accumulated into a flat fp32 arena whose views are the
parameters' ``.grad`` (use the optimizer's ``zero_grad`` to clear them).
"""
import torch
import torch.nn as nn

from .config import as_config
from .engine import Engine
from .norm import functional_l2_norm, functional_rms_norm, get_norm_fn
from .transformer_block import TransformerBlock
from .utils import trunc_normal_init_


class _GPTLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input_ids, labels, eng, anchor):
        A = eng.forward(input_ids, labels, training=True, want_loss=True, grad_scale=1.0)
        ctx.eng, ctx.acts = eng, A
        total = A.losses[0].clone()
        return total, A.losses[1].clone(), (A.losses[2] + A.losses[3]).clone()

    @staticmethod
    def backward(ctx, g_total, g_tok, g_q):
        # token / q losses are returned for logging; gradients flow through the total only
        ctx.eng.backward(ctx.acts, alpha_dev=g_total.reshape(1).float().contiguous())
        return None, None, None, None


class _GPTForward(torch.autograd.Function):
    """Reference-API forward: logits and q-head outputs are differentiable."""

    @staticmethod
    def forward(ctx, input_ids, labels, eng, anchor):
        A = eng.forward(input_ids, labels, training=True, want_loss=False)
        B, T = input_ids.shape
        ctx.eng, ctx.acts, ctx.shape = eng, A, (B, T)
        logits = A.logits.view(B, T, -1).clone()
        if eng._halting_active:
            import torch.nn.functional as F
            R = eng.n_recur
            lab = eng._labels
            correct = (A.argmax.long() == lab.view(1, -1)).float()  # [R, M]
            qh = A.q[..., 0]
            halt = F.binary_cross_entropy_with_logits(qh, correct, reduction="none").mean(dim=1).sum()
            qs = A.q.view(R, B, T, 2).clone()
            nxt = torch.maximum(qs[1:, ..., 0], qs[1:, ..., 1])
            targets = torch.sigmoid(torch.cat([nxt, qs[-1:, ..., 0]], dim=0))
            ctx.correct = correct
            ctx.mark_non_differentiable(targets)
            return logits, halt, qs, targets
        z = torch.zeros((), device=logits.device)
        ctx.mark_non_differentiable(z)
        return logits, z, z, z

    @staticmethod
    def backward(ctx, d_logits, d_halt, d_qs, d_targets):
        eng, A = ctx.eng, ctx.acts
        B, T = ctx.shape
        dl = d_logits.reshape(B * T, -1).to(torch.bfloat16).contiguous()
        if eng._halting_active:
            R = eng.n_recur
            M = B * T
            dq = torch.zeros(R, M, 2, device=dl.device, dtype=torch.float32)
            if d_qs is not None:
                dq += d_qs.reshape(R, M, 2).float()
            if d_halt is not None:
                dq[..., 0] += d_halt.float() * (torch.sigmoid(A.q[..., 0]) - ctx.correct) / M
            A.dq.copy_(dq)
        eng.backward(A, dlogits=dl)
        return None, None, None, None


class GPT(nn.Module):
    def __init__(self, **kwargs):
        super().__init__()
        config = as_config(kwargs)
        self.config = config
        self.name = config.name
        self.embs = nn.Embedding(config.vocab_size, config.d_model)
        self.dropout = nn.Dropout(config.dropout)
        self.layers = nn.ModuleList([TransformerBlock(config) for _ in range(config.n_layers)])
        self.norm_type = config.norm_type
        self.norm_eps = config.norm_eps
        if self.norm_type == "f_rmsnorm":
            self.ln_f = lambda x: functional_rms_norm(x, self.norm_eps)
        elif self.norm_type == "f_l2norm":
            self.ln_f = lambda x: functional_l2_norm(x, self.norm_eps)
        else:
            self.ln_f = get_norm_fn(config.norm_type, config.d_model, config.norm_eps)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        if config.get("n_recur", 1) > 1:
            self.q_head = nn.Linear(config.d_model, 2, bias=True)
        else:
            self.register_parameter("q_head", None)
        for name, module in self.named_modules():
            self._init_weights(module, name)
        self._engine = None

    def _init_weights(self, module, name=""):
        """Same init rules and RNG order as the reference (model/gpt.py:42-90)."""
        if isinstance(module, nn.Linear):
            if self.q_head is not None and module is self.q_head:
                with torch.no_grad():
                    module.weight.zero_()
                    module.bias.fill_(-5.0)
                return
            std, gain = 0.02, 1.0
            muon_routed = module.weight.ndim >= 2 and "embs" not in name and "lm_head" not in name
            if muon_routed:
                if hasattr(module, "RESIDUAL_SCALE_FLAG"):
                    gain *= (2 * self.config.n_layers) ** -0.5
                nn.init.xavier_uniform_(module.weight, gain=gain)
            else:
                if hasattr(module, "RESIDUAL_SCALE_FLAG"):
                    std *= (2 * self.config.n_layers) ** -0.5
                trunc_normal_init_(module.weight, std=std)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            trunc_normal_init_(module.weight, std=0.02)
        if hasattr(module, "attn_layer_scale"):
            with torch.no_grad():
                module.attn_layer_scale.fill_(0.1)
        if hasattr(module, "ff_layer_scale"):
            with torch.no_grad():
                module.ff_layer_scale.fill_(0.1)

    # ---------------------------------------------------------------- engine
    def engine(self) -> Engine:
        dev = self.lm_head.weight.device
        if self._engine is None or self._engine.device != dev:
            self._engine = Engine(self)
        return self._engine

    def _apply(self, fn, *args, **kwargs):
        # moving / casting parameters invalidates the engine's shadows and gradient arena
        self._engine = None
        return super()._apply(fn, *args, **kwargs)

    def _anchor(self):
        # a parameter input so autograd records the custom Functions as part of the graph
        return self.lm_head.weight

    # ---------------------------------------------------------------- API
    def forward(self, input_ids, labels=None):
        eng = self.engine()
        if torch.is_grad_enabled() and self.training:
            logits, halt, qs, targets = _GPTForward.apply(input_ids, labels, eng, self._anchor())
            if not eng._halting_active:
                return logits, halt, [], []
            return logits, halt, list(qs.unbind(0)), targets
        A = eng.forward(input_ids, labels, training=False, want_loss=False)
        B, T = input_ids.shape
        logits = A.logits.view(B, T, -1).clone()
        return logits, torch.zeros((), device=logits.device), [], []

    @torch.no_grad()
    def token_losses(self, input_ids, labels):
        """Per-token cross entropy [B, T] (fp32; 0 where labels == pad_token_id) of an eval-mode forward,
        e.g. to score the endings of a multiple-choice item."""
        eng = self.engine()
        A = eng.forward(input_ids, labels, training=False, want_loss=True)
        return A.loss_rows.view(input_ids.shape).clone()

    def forward_loss(self, input_ids, labels):
        """Fused forward + loss; returns (total, token, q) 0-d tensors, total differentiable."""
        eng = self.engine()
        if torch.is_grad_enabled() and self.training:
            return _GPTLoss.apply(input_ids, labels, eng, self._anchor())
        A = eng.forward(input_ids, labels, training=False, want_loss=True)
        return A.losses[0].clone(), A.losses[1].clone(), (A.losses[2] + A.losses[3]).clone()
