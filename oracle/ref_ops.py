"""CPU oracle for the rGPT training step. TEST INFRASTRUCTURE ONLY.

A plain fp32 (torch-on-CPU) restatement of the reference's algorithms
(newbee1905/rgpt), written functionally over a parameter dict that uses the
reference's parameter names. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import this module, and only as the checker or
the timed CPU baseline; the product path (rgpt_b200) never calls it.

Parity of this oracle is pinned against fixtures produced by running the
reference itself in the build container (tests/golden/gen_golden.py writes
tests/golden/*.pt; tests/test_oracle_golden.py checks this module against
them).

Reference file:line citations are relative to the reference repository root.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

# --------------------------------------------------------------------------
# Activations — model/kernels.py:13-118 (fp32 math)
# --------------------------------------------------------------------------
GELU_K = math.sqrt(2.0 / math.pi)  # model/kernels.py:19,30
GELU_C = 0.044715                   # model/kernels.py:20,35


def act_fwd(name: str, x: torch.Tensor) -> torch.Tensor:
    """f(x) for the four FFN activations (model/kernels.py:13-25,48-56,70-80,96-105)."""
    if name == "squared_relu":
        r = torch.clamp_min(x, 0.0)
        return r * r
    if name == "gelu":
        return 0.5 * x * (1.0 + torch.tanh(GELU_K * (x + GELU_C * x * x * x)))
    if name == "silu":
        return x * torch.sigmoid(x)
    if name == "mish":
        sp = torch.where(x > 20.0, x, torch.log(1.0 + torch.exp(x)))
        return x * torch.tanh(sp)
    return x


def act_grad(name: str, x: torch.Tensor) -> torch.Tensor:
    """f'(x) as written in the reference backward helpers (model/kernels.py:27-45,59-67,83-93,108-118)."""
    if name == "squared_relu":
        return 2.0 * torch.clamp_min(x, 0.0)
    if name == "gelu":
        x2 = x * x
        t = torch.tanh(GELU_K * (x + GELU_C * x2 * x))
        return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * (GELU_K * (1.0 + 3.0 * GELU_C * x2))
    if name == "silu":
        s = torch.sigmoid(x)
        return s * (1.0 + x * (1.0 - s))
    if name == "mish":
        sp = torch.where(x > 20.0, x, torch.log(1.0 + torch.exp(x)))
        t = torch.tanh(sp)
        return t + x * (1.0 - t * t) * torch.sigmoid(x)
    return torch.ones_like(x)


# --------------------------------------------------------------------------
# Fused linear + activation — model/kernels.py:289-374
# --------------------------------------------------------------------------
def linear_act_forward(x, w1, w2, act):
    """out = act(x @ w1^T) @ w2; returns (out, pre, post). w1 [N,K], w2 [N,Out] (model/kernels.py:291-331)."""
    pre = x @ w1.t()
    post = act_fwd(act, pre)
    return post @ w2, pre, post


def linear_act_backward(dy, x, w1, w2, pre, post, act):
    """(dx, dw1, dw2) of linear_act_forward (model/kernels.py:334-374)."""
    dw2 = post.t() @ dy
    dpre = (dy @ w2.t()) * act_grad(act, pre)
    dw1 = dpre.t() @ x
    dx = dpre @ w1
    return dx, dw1, dw2


# --------------------------------------------------------------------------
# Norms — model/norm.py
# --------------------------------------------------------------------------
def rmsnorm(x, weight, eps, add_unit_offset=True):
    """Gemma RMSNorm: x * rsqrt(mean(x^2) + eps), cast to the weight dtype, times (1 + w) (model/norm.py:21-34)."""
    var = (x * x).mean(dim=-1, keepdim=True)
    out = (x * torch.rsqrt(var + eps)).to(weight.dtype)
    return out * (1.0 + weight) if add_unit_offset else out * weight


def f_rmsnorm(x):
    """F.rms_norm over the last dim with eps = finfo(x.dtype).eps; the eps argument is ignored (model/norm.py:37-38)."""
    eps = torch.finfo(x.dtype).eps
    return x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps)


def hyperball(x):
    """x * rsqrt(1 + mean(x^2)) (model/norm.py:40-42, :160-162)."""
    return x * torch.rsqrt(1.0 + (x * x).mean(dim=-1, keepdim=True))


def l2norm(x, temp, eps):
    """x / (||x||_2 + eps) * temp (model/norm.py:50-51)."""
    return x / (torch.linalg.vector_norm(x, dim=-1, keepdim=True) + eps) * temp


def f_l2norm(x, eps):
    """x / (||x||_2 + eps) (model/norm.py:54-55)."""
    return x / (torch.linalg.vector_norm(x, dim=-1, keepdim=True) + eps)


def hybrid_elastic(x, alpha=0.5, eps=1e-6):
    """HybridElasticNorm (model/norm.py:83-95): s = sqrt(d) * rsqrt(max(sum x^2, eps)); scale = s if s < 1 else s^alpha."""
    d = x.shape[-1]
    sq = (x * x).sum(dim=-1, keepdim=True)
    hard = math.sqrt(d) * torch.rsqrt(sq.clamp_min(eps))
    return x * torch.where(hard < 1.0, hard, hard.pow(alpha))


def elastic_ball(x, alpha=0.5, eps=1e-6):
    """ElasticBallNorm (model/norm.py:118-132): scale = (sqrt(d) / sqrt(sum x^2 + eps))^alpha."""
    d = x.shape[-1]
    n = torch.sqrt((x * x).sum(dim=-1, keepdim=True) + eps)
    return x * (math.sqrt(d) / n).pow(alpha)


def norm_apply(kind, x, params, prefix, eps, d):
    """Dispatch a residual-stream / ln_f norm by config name (model/norm.py:165-179, model/gpt.py:25-30)."""
    if kind == "f_rmsnorm":
        return f_rmsnorm(x)
    if kind == "f_l2norm":
        return f_l2norm(x, eps)
    if kind == "rmsnorm":
        return rmsnorm(x, params[prefix + ".weight"], eps)
    if kind == "layernorm":
        return F.layer_norm(x, (d,), params[prefix + ".weight"], params[prefix + ".bias"], eps)
    if kind == "l2norm":
        return l2norm(x, params[prefix + ".temp"], eps)
    if kind == "elastic":
        return hybrid_elastic(x, 0.5, eps)
    if kind == "elasticball":
        return elastic_ball(x, 0.5, eps)
    if kind == "hyperball":
        return hyperball(x)
    return x


def qk_norm_apply(kind, q, k, params, prefix, eps, d_head):
    """QKNorm.forward (model/norm.py:182-204). The YAML alpha/scale keys never reach it
    (model/attention.py:25 passes only d_head, type, eps), so the defaults apply."""
    if kind in ("none",):
        return q, k
    if kind == "dual_elasticball":
        return elastic_ball(q, 0.5, eps), elastic_ball(k, 0.5, eps)
    if kind == "asymmetric_hyperball":
        return hyperball(q) * 1.0, hyperball(k) * 1.1
    return (norm_apply(kind, q, params, prefix + ".q_norm_fn", eps, d_head),
            norm_apply(kind, k, params, prefix + ".k_norm_fn", eps, d_head))


# --------------------------------------------------------------------------
# RoPE — model/rope.py:5-57 (non-interleaved rotate-half, base 10000)
# --------------------------------------------------------------------------
def rope_tables(T, d_head, base=10000.0, dtype=torch.float32):
    inv_freq = 1.0 / (base ** (torch.arange(0, d_head, 2).float() / d_head))  # model/rope.py:11
    t = torch.arange(T, dtype=dtype)                                           # model/rope.py:30
    freqs = torch.outer(t.float(), inv_freq).to(dtype)                        # model/rope.py:32
    emb = torch.cat((freqs, freqs), dim=-1)                                   # model/rope.py:33
    return emb.cos(), emb.sin()


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)  # model/rope.py:53-57


def rope_apply(q, k, cos, sin):
    """q*cos + rot(q)*sin for q, k in [B, H, T, D] (model/rope.py:38-51)."""
    return q * cos + rotate_half(q) * sin, k * cos + rotate_half(k) * sin


# --------------------------------------------------------------------------
# Attention — model/attention.py:35-64
# --------------------------------------------------------------------------
# --------------------------------------------------------------------------
# Dropout masks — nn.Dropout / SDPA dropout_p (model/gpt.py:96, model/transformer_block.py:45,52,
# model/attention.py:57). torch draws its own Philox stream, which no other implementation can
# reproduce bit for bit; the native kernels draw theirs from Philox4x32-10 with the counter layout
# below, and this restatement regenerates exactly those masks so that a dropout step can be checked
# element by element. Philox4x32-10: Salmon, Moraes, Dror and Shaw, SC 2011 (checked against the
# published known-answer vectors in tests/test_oracle_golden.py).
# --------------------------------------------------------------------------
_U32 = np.uint64(0xFFFFFFFF)
EMB_DROP_SITE = 0xFFFFFF


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32-10 over uint32 counter arrays; returns the four output words (uint32)."""
    c = [np.asarray(x, dtype=np.uint64) for x in np.broadcast_arrays(c0, c1, c2, c3)]
    k0, k1 = np.uint64(k0), np.uint64(k1)
    for _ in range(10):
        p0 = np.uint64(0xD2511F53) * c[0]
        p1 = np.uint64(0xCD9E8D57) * c[2]
        c = [(p1 >> np.uint64(32)) ^ c[1] ^ k0, p1 & _U32, (p0 >> np.uint64(32)) ^ c[3] ^ k1, p0 & _U32]
        k0 = (k0 + np.uint64(0x9E3779B9)) & _U32
        k1 = (k1 + np.uint64(0xBB67AE85)) & _U32
    return [x.astype(np.uint32) for x in c]


def drop_thresh(p):
    """Keep iff a 16-bit uniform >= round(p * 65536)."""
    return int(round(p * 65536.0))


def keep_mask(seed, site, sub, rows, cols, p):
    """Keep mask [rows, cols] (bool): element (r, c) is 16-bit half (c & 1) of word (c >> 1) & 3 of
    Philox block (c >> 3, r, site, sub) under key (seed low 32 bits, seed high 32 bits)."""
    cb = (cols + 7) // 8
    r = np.arange(rows, dtype=np.uint64)[:, None]
    b = np.arange(cb, dtype=np.uint64)[None, :]
    w = philox4x32_10(b, r, np.uint64(site), np.uint64(sub), seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    w = np.stack(w, axis=-1)                                   # [rows, cb, 4]
    halves = np.stack([w & 0xFFFF, w >> 16], axis=-1)          # [rows, cb, 4, 2]
    u16 = halves.reshape(rows, cb * 8)[:, :cols]
    return torch.from_numpy(u16 >= drop_thresh(p))


def resid_drop_mask(seed, site, M, d, p):
    """Residual-branch / embedding mask over [M, d] (rows = tokens), sub-stream 0."""
    return keep_mask(seed, site, 0, M, d, p)


def attn_drop_mask(seed, site, B, H, T, p):
    """Attention-probability mask [B, H, T(query), T(key)]: head bh = b*H + h is sub-stream bh."""
    return torch.stack([keep_mask(seed, site, bh, T, T, p) for bh in range(B * H)]).view(B, H, T, T)


def causal_attention(q, k, v, scale, keep=None, p=0.0):
    """softmax(q k^T * scale + causal mask) v, q/k/v [B, H, T, D] (F.scaled_dot_product_attention, is_causal).

    keep: optional [B, H, T, T] dropout mask applied to the probabilities (scaled by 1/(1-p))."""
    T = q.shape[-2]
    s = (q @ k.transpose(-2, -1)) * scale
    mask = torch.ones(T, T, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    pr = torch.softmax(s, dim=-1)
    if keep is not None:
        pr = pr * keep.to(pr.dtype) * (1.0 / (1.0 - p))
    return pr @ v


def attention_forward(x, params, prefix, cfg, drop=None):
    B, T, d = x.shape
    H = cfg["n_heads"]
    Dh = d // H
    q = (x @ params[prefix + ".q_proj.weight"].t()).view(B, T, H, Dh)
    k = (x @ params[prefix + ".k_proj.weight"].t()).view(B, T, H, Dh)
    v = (x @ params[prefix + ".v_proj.weight"].t()).view(B, T, H, Dh)
    qk = cfg.get("qk_normtype", "f_rmsnorm")
    if qk != "none":
        q, k = qk_norm_apply(qk, q, k, params, prefix + ".qk_norm", cfg["norm_eps"], Dh)
    gate = None
    if cfg.get("g1_gate", False):  # model/attention.py:45-48: one Linear(d_head, d_head) shared by every head
        gate = torch.sigmoid(q @ params[prefix + ".gate_proj.weight"].t() + params[prefix + ".gate_proj.bias"])
        gate = gate.transpose(1, 2)
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    cos, sin = rope_tables(T, Dh, 10000.0, q.dtype)
    q, k = rope_apply(q, k, cos, sin)
    keep = None
    if drop is not None:
        if drop["seed"] == "torch":  # torch's own generator, as the reference draws it (timing only)
            keep = torch.rand(B, H, T, T) >= drop["p"]
        else:
            keep = attn_drop_mask(drop["seed"], drop["site"] + 2, B, H, T, drop["p"])
    o = causal_attention(q, k, v, 1.0 / math.sqrt(Dh), keep, drop["p"] if drop else 0.0)
    if gate is not None:
        o = o * gate
    o = o.transpose(1, 2).reshape(B, T, d)
    return o @ params[prefix + ".out_proj.weight"].t()


def _dropped(y, drop, site):
    """nn.Dropout with the native kernels' mask of `site` over the rows of y [B, T, d]."""
    if drop is None:
        return y
    if drop["seed"] == "torch":  # torch's own dropout, as the reference runs it (timing only)
        return F.dropout(y, drop["p"], training=True)
    B, T, d = y.shape
    keep = resid_drop_mask(drop["seed"], site, B * T, d, drop["p"]).view(B, T, d)
    return y * keep.to(y.dtype) * (1.0 / (1.0 - drop["p"]))


def block_forward(x, params, prefix, cfg, drop=None):
    """Pre-norm block with optional layer scale (model/transformer_block.py:43-57).

    drop: None (dropout off) or {"p", "seed", "site"}: branch masks at sites site+0 (attention
    output) and site+1 (FFN output), the attention-probability mask at site+2."""
    d = cfg["d_model"]
    nt, eps = cfg["norm_type"], cfg["norm_eps"]
    a = attention_forward(norm_apply(nt, x, params, prefix + ".attn_norm", eps, d), params, prefix + ".attn", cfg,
                          drop)
    a = _dropped(a, drop, drop["site"] if drop else 0)
    h = x + (a * params[prefix + ".attn_layer_scale"] if cfg.get("use_layer_scale") else a)
    hn = norm_apply(nt, h, params, prefix + ".ff_norm", eps, d)
    B, T, _ = hn.shape
    f, _, _ = linear_act_forward(hn.reshape(-1, d), params[prefix + ".ff.fc1.weight"],
                                 params[prefix + ".ff.fc2.weight"].t(), cfg["activation_type"])
    f = _dropped(f.view(B, T, d), drop, drop["site"] + 1 if drop else 0)
    return h + (f * params[prefix + ".ff_layer_scale"] if cfg.get("use_layer_scale") else f)


def gpt_forward(params, input_ids, cfg, labels=None, training=True, drop_seed=None):
    """GPT.forward (model/gpt.py:92-143).

    Dropout is off unless drop_seed is given (with training and cfg["dropout"] > 0): then the
    embedding output uses site EMB_DROP_SITE and layer application `app` (recurrence i, layer li,
    app = i * n_layers + li) sites 4 * app + {0, 1, 2}, the masks of the native kernels.
    drop_seed="torch" draws the masks from torch's generator instead, as the reference does; only
    the timed CPU baseline uses it (its masks cannot be compared with anything).
    Returns (final_logits, accum_halt_loss, all_step_q, target_q_continues)."""
    d = cfg["d_model"]
    nt, eps = cfg["norm_type"], cfg["norm_eps"]
    p = cfg.get("dropout", 0.0)
    use_drop = training and drop_seed is not None and p > 0
    x = params["embs.weight"][input_ids]
    if use_drop:
        x = _dropped(x, {"p": p, "seed": drop_seed}, EMB_DROP_SITE)
    n_recur = cfg.get("n_recur", 1)
    all_q = []
    halt = torch.zeros(())
    for i in range(n_recur):
        for li in range(cfg["n_layers"]):
            drop = {"p": p, "seed": drop_seed, "site": 4 * (i * cfg["n_layers"] + li)} if use_drop else None
            x = block_forward(x, params, f"layers.{li}", cfg, drop)
        if cfg.get("cal_halt_loss") and labels is not None:
            h = norm_apply(nt, x, params, "ln_f", eps, d)
            cur_q = h @ params["q_head.weight"].t() + params["q_head.bias"]
            all_q.append(cur_q)
            step_logits = h @ params["lm_head.weight"].t()  # its CE is computed then dropped (model/gpt.py:113-117)
            with torch.no_grad():
                correct = (step_logits.argmax(dim=-1) == labels).float().unsqueeze(-1)
            halt = halt + F.binary_cross_entropy_with_logits(cur_q[..., 0:1], correct)
        if cfg.get("detach_recur") and i < n_recur - 1:
            x = x.detach()
    logits = norm_apply(nt, x, params, "ln_f", eps, d) @ params["lm_head.weight"].t()
    targets = []
    if training and n_recur > 1 and all_q:
        with torch.no_grad():
            qs = torch.stack(all_q, dim=0)
            nxt = torch.maximum(qs[1:, ..., 0], qs[1:, ..., 1])
            targets = torch.sigmoid(torch.cat([nxt, qs[-1:, ..., 0]], dim=0))
    return logits, halt, all_q, targets


def compute_loss(outputs, labels, ignore_index=-100):
    """Trainer.compute_loss (trainer.py:139-167): token CE + mean BCE(q_continue, target) + mean halt loss."""
    logits, halt, all_q, targets = outputs
    token = F.cross_entropy(logits.reshape(-1, logits.size(-1)), labels.reshape(-1), ignore_index=ignore_index)
    q_cont = torch.zeros(())
    if len(all_q) > 0:
        for i, q in enumerate(all_q):
            q_cont = q_cont + F.binary_cross_entropy_with_logits(q[..., 1], targets[i])
        q_cont = q_cont / len(all_q)
    avg_halt = halt / len(all_q) if len(all_q) > 0 else 0.0
    return token + q_cont + avg_halt, token


# --------------------------------------------------------------------------
# Optimizer — optimizer.py
# --------------------------------------------------------------------------
NS_COEFFS = (3.4445, -4.7750, 2.0315)  # optimizer.py:19


def zeropower_ns5(G, steps=5, coeffs=NS_COEFFS, dtype=torch.bfloat16):
    """Quintic Newton-Schulz (optimizer.py:8-45).

    dtype=torch.bfloat16 keeps the reference's bf16 rounding after every op;
    dtype=torch.float32 is the exact-arithmetic restatement used for the 1e-3 bar."""
    a, b, c = coeffs
    X = G.to(dtype)
    transposed = X.size(-2) > X.size(-1)
    if transposed:
        X = X.transpose(-2, -1)
    X = X.contiguous()
    nrm = X.float().norm(dim=(-2, -1), keepdim=True).clamp_min(1e-7)
    X = (X.float() / nrm).to(dtype)
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        A2 = A @ A
        Bm = torch.add(b * A, A2, alpha=c)
        X = torch.add(a * X, Bm @ X)
    if transposed:
        X = X.transpose(-2, -1)
    return X


def muon_scale(m, n):
    """sqrt(max(1, m/n)) (optimizer.py:130-133)."""
    r = m / n
    return math.sqrt(r) if r > 1.0 else 1.0


def muon_update(grad, momentum, beta=0.95, ns_steps=5, nesterov=True, scale=1.0, ns_dtype=torch.bfloat16):
    """optimizer.py:51-74. Updates `momentum` (bf16) in place; returns the bf16 update."""
    g = grad.to(momentum.dtype)
    momentum.lerp_(g, 1.0 - beta)
    g = g.lerp_(momentum, beta) if nesterov else momentum
    upd = zeropower_ns5(g, steps=ns_steps, dtype=ns_dtype).to(momentum.dtype)
    if scale != 1.0:
        upd = upd * scale
    return upd


def adamw_step(params, grads, exp_avgs, exp_avg_sqs, step, lr, wd, beta1, beta2, eps):
    """foreach_adamw_step restated per tensor (optimizer.py:80-116); updates in place."""
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    for p, g, m, v in zip(params, grads, exp_avgs, exp_avg_sqs):
        if wd != 0.0:
            p.mul_(1.0 - lr * wd)
        m.lerp_(g, 1.0 - beta1)
        v.lerp_(g * g, 1.0 - beta2)
        denom = v.sqrt() * (1.0 / math.sqrt(bc2)) + eps
        p.add_((m / denom) * (1.0 / bc1), alpha=-lr)


def param_groups(named_params, tie_word_embeddings=False):
    """Trainer's Muon / AdamW-decay / AdamW-no-decay split (trainer.py:66-95). Returns three name lists."""
    muon, decay, no_decay = [], [], []
    for name, p in named_params:
        if not tie_word_embeddings and "lm_head" in name:
            decay.append(name)
        elif "emb" in name:
            no_decay.append(name)
        elif p.ndim >= 2:
            muon.append(name)
        elif "norm" in name or "bias" in name:
            no_decay.append(name)
        else:
            decay.append(name)
    return muon, decay, no_decay


class OracleMuon:
    """Muon.step (optimizer.py:181-272) over a name->tensor dict, with the Trainer's groups."""

    def __init__(self, params, lr=6e-4, weight_decay=0.1, momentum=0.95, nesterov=True,
                 adam_betas=(0.9, 0.95), adam_eps=1e-8, muon_lr_multiplier=33.3, ns_steps=5,
                 tie_word_embeddings=False, ns_dtype=torch.bfloat16):
        self.params = params
        self.lr, self.wd = lr, weight_decay
        self.beta, self.nesterov = momentum, nesterov
        self.betas, self.eps = adam_betas, adam_eps
        self.mult, self.ns_steps = muon_lr_multiplier, ns_steps
        self.ns_dtype = ns_dtype
        self.groups = param_groups(list(params.items()), tie_word_embeddings)
        self.state = {}
        self.adam_steps = [0, 0]

    @torch.no_grad()
    def step(self, grads, lr=None):
        lr = self.lr if lr is None else lr
        muon, decay, no_decay = self.groups
        for name in muon:
            p, g = self.params[name], grads.get(name)
            if g is None:
                continue
            st = self.state.setdefault(name, {"momentum_buffer": torch.zeros_like(p, dtype=torch.bfloat16)})
            if self.wd != 0.0:
                p.mul_(1.0 - lr * self.wd)
            g2 = g.view(g.size(0), -1)
            m2 = st["momentum_buffer"].view(g.size(0), -1)
            upd = muon_update(g2, m2, self.beta, self.ns_steps, self.nesterov,
                              muon_scale(g2.size(0), g2.size(1)), self.ns_dtype)
            p.add_(upd.view_as(p).float(), alpha=-lr * self.mult)
        for gi, (names, wd) in enumerate(((decay, self.wd), (no_decay, 0.0))):
            live = [n for n in names if grads.get(n) is not None]
            if not live:
                continue
            self.adam_steps[gi] += 1
            for n in live:
                self.state.setdefault(n, {"exp_avg": torch.zeros_like(self.params[n]),
                                          "exp_avg_sq": torch.zeros_like(self.params[n])})
            adamw_step([self.params[n] for n in live], [grads[n] for n in live],
                       [self.state[n]["exp_avg"] for n in live], [self.state[n]["exp_avg_sq"] for n in live],
                       self.adam_steps[gi], lr, wd, self.betas[0], self.betas[1], self.eps)


def train_steps(params, cfg, batches, n_steps, opt_kwargs=None, lr_schedule=None):
    """Trainer step body (trainer.py:182-224) in fp32, dropout off, grad_accum = len(batch list per step).

    `batches` yields lists of (input_ids, labels) micro-batches. Returns the per-step total losses."""
    params = {k: v.clone().requires_grad_(True) for k, v in params.items()}
    opt = OracleMuon(params, **(opt_kwargs or {}))
    losses = []
    it = iter(batches)
    for s in range(n_steps):
        micro = next(it)
        grads = {}
        total = 0.0
        for ids, labels in micro:
            out = gpt_forward(params, ids[:, :-1], cfg, labels=labels[:, 1:].contiguous(), training=True)
            loss, _ = compute_loss(out, labels[:, 1:])
            loss = loss / len(micro)
            gs = torch.autograd.grad(loss, [params[k] for k in params], allow_unused=True)
            for k, g in zip(params, gs):
                if g is not None:
                    grads[k] = grads[k] + g if k in grads else g
            total += loss.item()
        lr = lr_schedule(s) if lr_schedule else None
        opt.step(grads, lr=lr)
        losses.append(total)
    return losses, {k: v.detach() for k, v in params.items()}
