"""Generate golden fixtures by running the reference implementation itself.

Runs only in the build container, where the reference checkout is mounted at
/root/reference (read-only). It imports the reference's own modules with two
shims: a minimal `omegaconf`/`hydra` stand-in (neither is installed here) and
eager execution (TORCHDYNAMO_DISABLE=1; torch.compile cannot build on this CPU
box). The fused Triton FFN kernels run under TRITON_INTERPRET=1, with
libdevice.tanh replaced by the identity tanh(x) = 2*sigmoid(2x) - 1 because
the interpreter cannot call libdevice.

Outputs tests/golden/*.pt (small, CPU fp32). tests/test_oracle_golden.py checks
the oracle against them; GPU parity tests use them as fixed inputs/outputs.

    RGPT_REFERENCE=<reference checkout> python tests/golden/gen_golden.py [fixture ...]

The reference checkout defaults to /root/reference; with no fixture names every
fixture is regenerated.
"""
import os
import sys
import types

os.environ["TORCHDYNAMO_DISABLE"] = "1"
os.environ["TRITON_INTERPRET"] = "1"

REF = os.environ.get("RGPT_REFERENCE", "/root/reference")
OUT = os.path.dirname(os.path.abspath(__file__))


def install_shims():
    class DictConfig(dict):
        def __getattr__(self, k):
            try:
                return self[k]
            except KeyError as e:
                raise AttributeError(k) from e

    class OmegaConf:
        @staticmethod
        def to_yaml(cfg):
            return str(cfg)

        @staticmethod
        def set_struct(cfg, flag):
            return None

    om = types.ModuleType("omegaconf")
    om.DictConfig = DictConfig
    om.OmegaConf = OmegaConf
    sys.modules["omegaconf"] = om
    hy = types.ModuleType("hydra")
    hy.core = types.SimpleNamespace(hydra_config=types.SimpleNamespace(HydraConfig=None))
    hy.main = lambda **kw: (lambda f: f)
    sys.modules["hydra"] = hy
    ds = types.ModuleType("datasets")  # dataset.py imports it at module level; nothing here downloads

    def _no_download(*a, **k):
        raise RuntimeError("no dataset downloads in the golden generator")

    ds.load_dataset = _no_download
    sys.modules.setdefault("datasets", ds)
    sys.path.insert(0, REF)


install_shims()

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

from model.gpt import GPT  # noqa: E402
from model.attention import Attention  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _tanh_for_interpreter(x):
    # triton 3.6's interpreter has no libdevice.tanh; tanh(x) = 2*sigmoid(2x) - 1 exactly
    # (differs from libdevice by float rounding only, ~1e-7).
    return 2.0 * tl.sigmoid(2.0 * x) - 1.0


tl.extra.cuda.libdevice.tanh = _tanh_for_interpreter

from model.kernels import FusedLinearActivationFunction  # noqa: E402
from model import norm as rnorm  # noqa: E402
from model.rope import RotaryEmbedding  # noqa: E402
import optimizer as ropt  # noqa: E402
from trainer import Trainer  # noqa: E402

ACTS = ["squared_relu", "gelu", "silu", "mish"]


def eager(fn):
    return getattr(fn, "_torchdynamo_orig_callable", fn)


def save(name, obj):
    path = os.path.join(OUT, name)
    torch.save(obj, path)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


def gen_ffn():
    torch.manual_seed(42)
    M, N, K, Out = 64, 128, 64, 32
    x = torch.randn(M, K) * 0.1
    w1 = torch.randn(N, K) * 0.1
    w2 = torch.randn(N, Out) * 0.1
    res = {"x": x, "w1": w1, "w2": w2}
    for act in ACTS:
        xx, a, b = (t.clone().requires_grad_(True) for t in (x, w1, w2))
        y = FusedLinearActivationFunction.apply(xx, a, b, act)  # the Triton kernels, interpreted on CPU
        y.sum().backward()
        res[act] = {"y": y.detach(), "dx": xx.grad, "dw1": a.grad, "dw2": b.grad}
    save("ffn.pt", res)


def gen_norms():
    torch.manual_seed(1)
    x = torch.randn(3, 5, 64) * 1.7
    x[0, 0] *= 0.01  # a short row, so HybridElasticNorm takes its elastic branch
    g = torch.randn(3, 5, 64)
    res = {"x": x, "g": g}
    mods = {
        "rmsnorm": rnorm.RMSNorm(64, 1e-5),
        "l2norm": rnorm.L2Norm(64, 1e-5),
        "elastic": rnorm.HybridElasticNorm(64, eps=1e-5),
        "elasticball": rnorm.ElasticBallNorm(64, eps=1e-5),
        "hyperball": rnorm.HyperballNorm(),
    }
    with torch.no_grad():
        mods["rmsnorm"].weight.normal_(0, 0.3)
        mods["l2norm"].temp.fill_(1.3)
    for name, m in mods.items():
        xx = x.clone().requires_grad_(True)
        y = m(xx)
        (y * g).sum().backward()
        entry = {"y": y.detach(), "dx": xx.grad}
        for pn, p in m.named_parameters():
            entry["param_" + pn] = p.detach().clone()
            entry["grad_" + pn] = p.grad.clone()
        res[name] = entry
    for name, fn in {"f_rmsnorm": lambda t: rnorm.functional_rms_norm(t, 1e-5),
                     "f_l2norm": lambda t: rnorm.functional_l2_norm(t, 1e-5)}.items():
        xx = x.clone().requires_grad_(True)
        y = fn(xx)
        (y * g).sum().backward()
        res[name] = {"y": y.detach(), "dx": xx.grad}
    save("norms.pt", res)


def gen_rope_attention():
    torch.manual_seed(2)
    rope = RotaryEmbedding(32, max_seq_len=64)
    q = torch.randn(2, 3, 20, 32)
    k = torch.randn(2, 3, 20, 32)
    qo, ko = rope(q, k)
    res = {"q": q, "k": k, "q_out": qo, "k_out": ko}
    cfg = dict(n_heads=4, d_model=64, g1_gate=True, qk_normtype="f_rmsnorm", norm_eps=1e-5, max_seq_len=64,
               dropout=0.0)
    DictConfig = sys.modules["omegaconf"].DictConfig
    attn = Attention(DictConfig(cfg))
    for p in attn.parameters():
        if p.ndim == 2:
            torch.nn.init.xavier_uniform_(p)
    x = torch.randn(2, 24, 64, requires_grad=True)
    y = attn(x)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    res["attn"] = {"cfg": cfg, "state": {k: v.detach().clone() for k, v in attn.state_dict().items()},
                   "x": x.detach(), "y": y.detach(), "gy": gy, "dx": x.grad,
                   "grads": {n: p.grad.clone() for n, p in attn.named_parameters()}}
    save("rope_attention.pt", res)


TINY = dict(name="gpt", n_layers=2, n_recur=1, detach_recur=False, cal_halt_loss=False, n_heads=2, d_model=32,
            vocab_size=64, max_seq_len=32, dropout=0.0, norm_type="rmsnorm", norm_eps=1e-5,
            qk_normtype="f_rmsnorm", activation_type="squared_relu", g1_gate=True, use_layer_scale=False,
            pad_token_id=-100, tie_word_embeddings=False)
TINY_RGPT = dict(TINY, name="rgpt", n_layers=1, n_recur=3, cal_halt_loss=True, use_layer_scale=True)
TINY_ELASTIC = dict(TINY, qk_normtype="elastic", use_layer_scale=True, activation_type="gelu")


def loss_of(outputs, labels):
    stub = types.SimpleNamespace(criterion=torch.nn.CrossEntropyLoss(ignore_index=-100), device=torch.device("cpu"))
    out = Trainer.compute_loss(stub, outputs, labels)
    return out if isinstance(out, torch.Tensor) else out[0]


def gen_model(tag, cfg, seed):
    torch.manual_seed(seed)
    model = GPT(**cfg)
    model.train()
    B, T = 2, 17
    ids = torch.randint(0, cfg["vocab_size"], (B, T + 1))
    ids[1, -3:] = torch.randint(0, cfg["vocab_size"], (3,))
    labels = ids.clone()
    labels[0, 5] = -100  # one ignored position
    inp, tgt = ids[:, :-1], labels[:, 1:].contiguous()
    outputs = model(inp, labels=tgt)
    loss = loss_of(outputs, labels[:, 1:])
    loss.backward()
    logits, halt, qs, targets = outputs
    save(f"model_{tag}.pt", {
        "cfg": cfg, "seed": seed,
        "state": {k: v.detach().clone() for k, v in model.state_dict().items()},
        "ids": ids, "labels": labels,
        "logits": logits.detach(), "halt": halt.detach(),
        "qs": [q.detach() for q in qs], "targets": targets if isinstance(targets, list) else targets.detach(),
        "loss": loss.detach(),
        "grads": {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None},
    })


def gen_optim():
    torch.manual_seed(3)
    ns = eager(ropt.zeropower_via_newtonschulz5)
    mu = eager(ropt.muon_update)
    res = {}
    for shape in [(48, 32), (32, 80), (64, 64)]:
        G = torch.randn(*shape) * 0.01
        res[f"ns_{shape[0]}x{shape[1]}"] = {"G": G, "X": ns(G, 5).float()}
    G1 = torch.randn(96, 32) * 0.01
    G2 = torch.randn(96, 32) * 0.01
    m = torch.zeros(96, 32, dtype=torch.bfloat16)
    u1 = mu(G1, m, beta=0.95, ns_steps=5, nesterov=True, scale=ropt._muon_scale(96, 32)).float()
    m1 = m.clone()
    u2 = mu(G2, m, beta=0.95, ns_steps=5, nesterov=True, scale=ropt._muon_scale(96, 32)).float()
    res["muon"] = {"G1": G1, "G2": G2, "u1": u1, "m1": m1.float(), "u2": u2, "m2": m.float()}
    ps = [torch.randn(512) * 0.01 + 1.0, torch.randn(7, 9)]
    gs_steps = [[torch.randn_like(p) * 1e-3 for p in ps] for _ in range(3)]
    p_run = [p.clone() for p in ps]
    m1s = [torch.zeros_like(p) for p in ps]
    m2s = [torch.zeros_like(p) for p in ps]
    for s, gs in enumerate(gs_steps):
        ropt.foreach_adamw_step(p_run, gs, m1s, m2s, step=s + 1, lr=0.02, wd=0.1, beta1=0.9, beta2=0.95, eps=1e-8)
    res["adamw"] = {"p0": ps, "grads": gs_steps, "p3": p_run, "m": m1s, "v": m2s}
    save("optim.pt", res)


def gen_train(tag, cfg, seed, n_steps, accum):
    torch.manual_seed(seed)
    model = GPT(**cfg)
    model.train()
    init = {k: v.detach().clone() for k, v in model.state_dict().items()}
    muon, dec, nodec = [], [], []
    for name, p in model.named_parameters():  # trainer.py:66-95
        if "lm_head" in name:
            dec.append(p)
        elif "emb" in name:
            nodec.append(p)
        elif p.ndim >= 2:
            muon.append(p)
        elif "norm" in name or "bias" in name:
            nodec.append(p)
        else:
            dec.append(p)
    groups = [{"params": muon, "use_muon": True}, {"params": dec, "use_muon": False, "weight_decay": 0.1},
              {"params": nodec, "use_muon": False, "weight_decay": 0.0}]
    opt = ropt.Muon(groups, lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    gen = torch.Generator().manual_seed(seed + 100)
    batches = [[torch.randint(0, cfg["vocab_size"], (2, 17), generator=gen) for _ in range(accum)]
               for _ in range(n_steps)]
    losses = []
    for micro in batches:  # trainer.py:182-224 (fp32: no autocast, no scaler)
        tot = 0.0
        for ids in micro:
            out = model(ids[:, :-1], labels=ids[:, 1:].contiguous())
            loss = loss_of(out, ids[:, 1:]) / accum
            loss.backward()
            tot += loss.item()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(tot)
    save(f"train_{tag}.pt", {"cfg": cfg, "init": init, "batches": batches, "losses": losses,
                             "final": {k: v.detach().clone() for k, v in model.state_dict().items()}})


class ToyTokenizer:
    """A deterministic stand-in for a GPT-2 tokenizer: one id per character. No pad token, so the
    collate falls back to EOS for padding, as it does with GPT-2."""

    pad_token_id = None
    eos_token_id = 1
    bos_token_id = 2

    def encode(self, text, add_special_tokens=True):
        return [3 + (ord(c) % 97) for c in text]


# synthetic multiple-choice items (invented strings, not HellaSwag's)
MC_ITEMS = [
    {"context": "the cat sat on", "endings": ["the mat", "a hat", "the moon and stars", "x"], "label": 0},
    {"context": "numbers go up by one: 1 2 3", "endings": [" 4", " 9", " 4 5 6 7 8 9 10", ""], "label": 0},
    {"context": "a long context " * 3, "endings": ["ends here", "or there", "maybe", "never"], "label": 3},
]


def gen_hellaswag_collate():
    from dataset import hellaswag_collate_fn  # the reference's collate (dataset.py:71-153)

    out = hellaswag_collate_fn(MC_ITEMS, ToyTokenizer(), max_seq_len=24)
    save("hellaswag_collate.pt", {"items": MC_ITEMS, "max_seq_len": 24, "out": out})


GENERATORS = {
    "ffn": gen_ffn, "norms": gen_norms, "rope_attention": gen_rope_attention,
    "model_gpt": lambda: gen_model("gpt", TINY, 11), "model_rgpt": lambda: gen_model("rgpt", TINY_RGPT, 12),
    "model_elastic": lambda: gen_model("elastic", TINY_ELASTIC, 13), "optim": gen_optim,
    "train_gpt": lambda: gen_train("gpt", TINY, 21, 6, 1), "train_rgpt": lambda: gen_train("rgpt", TINY_RGPT, 22, 4, 2),
    "hellaswag_collate": gen_hellaswag_collate,
}

if __name__ == "__main__":
    for name in sys.argv[1:] or list(GENERATORS):
        GENERATORS[name]()
