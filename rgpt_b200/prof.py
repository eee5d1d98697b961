"""One launch of each hot kernel of the gpt-small training step, for profiler captures.

    python -m rgpt_b200.prof

Runs, once each and in this order, on cuda:0 with seeded random inputs at the gpt-small
sizes (16 x 1024 tokens, d_model 512, 8 heads, FFN 2048, vocabulary 50304):
  1. weight-gradient GEMM  dW1 += dpre^T hn2  (2048 x 512, K = 16384; CTA-pair tiles, split-K
     bulk reduce-add)
  2. input-gradient GEMM   dX = dlogits W     (16384 x 512, K = 8192, W read MN-major; CTA pairs)
  3. QKV projection GEMM   qkv = x Wqkv^T     (16384 x 1536, K = 512; single-CTA tiles)
  4. causal attention forward   (B 16, T 1024, H 8, head dim 64)
  5. causal attention backward  (same sizes; after its bf16-gate prep kernel)
  6. cross entropy with the gradient written in place (4096 rows x 50304)
  7. lm_head forward GEMM  logits = h Wlm^T  (4096 x 50304, K = 512; CTA pairs, bf16 store)
  8. G1 gate GEMM          gate = sigmoid(q_n Wg^T + bg)  (131072 x 64, K = 64; bias+sigmoid epilogue)
Device memory stays under 2 GB, so a multi-pass profiler capture saves and restores little.

    python -m rgpt_b200.prof bw

runs instead the bandwidth-bound kernels and the optimizer of the same step, once each:
  rownorm forward / backward (16384 x 512), QKV prep forward / backward (QK-norm + RoPE + gate
  input), attention backward prep, embedding forward / backward, cross entropy over all 16384 rows,
  then one Muon + AdamW step over the gpt-small parameter shapes (AdamW over 51.5 M parameters;
  Muon: momentum/transposition, the batched Newton-Schulz GEMMs of the [512, 512] x 32 and
  [512, 2048] x 16 classes, apply), one fp32 Newton-Schulz iteration of one [512, 2048] matrix,
  and the dropout-0.1 variants of the attention forward and the residual GEMM. Device memory stays
  under 3 GB.

    python -m rgpt_b200.prof ffn

times the fused linear+activation sweep (forward + backward, M in {8192 .. 65536}, four activations)
with CUDA events and prints a table.
"""
import sys

import torch

from rgpt_b200 import native as nv


def main() -> None:
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(0)
    def rb(*shape):
        return torch.randn(*shape, device=dev, generator=g).bfloat16()

    M, d, F, V = 16384, 512, 2048, 50304
    # 1 weight-gradient GEMM (CTA pair, split-K reduce-add): dW1 += dpre^T hn2   [2048 x 512, K = 16384]
    dpre, hn2 = rb(M, F), rb(M, d)
    dw1 = torch.zeros(F, d, device=dev)
    nv.gemm(dpre.t(), hn2.t(), dw1, epi=nv.EPI_ACCUM_F32, splitk=0)
    # 2 lm_head-style input gradient (CTA pair, B MN-major): dX = dlogits W   [16384 x 512, K = 8192]
    dl, W = rb(M, 8192), rb(8192, d)
    dx = torch.empty(M, d, device=dev)
    nv.gemm(dl, W.t(), dx, epi=nv.EPI_STORE_F32)
    torch.cuda.synchronize(); del dl, W, dpre; torch.cuda.empty_cache()
    # 3 QKV projection (single-CTA tiles, K = 512)
    x, wqkv = rb(M, d), rb(3 * d, d)
    qkv = torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16)
    nv.gemm(x, wqkv, qkv)
    # 4/5 attention forward and backward (B=16, T=1024, H=8)
    B, T, H = 16, 1024, 8
    qk = rb(M, 2 * d); gate = torch.sigmoid(torch.randn(M, d, device=dev, generator=g)).bfloat16()
    o = torch.empty(M, d, device=dev, dtype=torch.bfloat16); og = torch.empty_like(o)
    lse = torch.empty(B, H, T, device=dev)
    nv.attn_fwd(qk, qkv, gate, o, og, lse, B, T, H)
    dog = rb(M, d); do = torch.empty_like(o); dgp = torch.empty_like(o); D = torch.empty(B, H, T, device=dev)
    nv.attn_bwd_prep(dog, o, gate, do, dgp, D, B, T, H)
    dq = torch.zeros(M, d, device=dev); dk = torch.empty(M, d, device=dev)
    dqkv = torch.zeros(M, 3 * d, device=dev, dtype=torch.bfloat16)
    nv.attn_bwd(qk, qkv, do, lse, D, dq, dk, dqkv[:, 2 * d:], B, T, H)
    # 6 cross entropy over the vocabulary (row in shared memory), with the gradient written in place
    Mc = 4096
    logits = rb(Mc, V)
    labels = torch.randint(0, V, (Mc,), device=dev, generator=g)
    rows = torch.empty(Mc, device=dev); sb = torch.empty(4, device=dev); lo = torch.empty(1, device=dev)
    nv.cross_entropy(logits, labels, loss_rows=rows, scale_buf=sb, loss_out=lo, write_grad=True)
    # 7 lm_head forward into bf16 logits (the same 4096 x 50304 buffer)
    h, wlm = rb(Mc, d), rb(V, d)
    nv.gemm(h, wlm, logits)
    # 8 G1 gate of every (token, head): [M*H, 64] x [64, 64]^T, bias + sigmoid epilogue
    qn, wg = rb(M * H, 64), rb(64, 64)
    bg = torch.randn(64, device=dev, generator=g)
    gate_out = torch.empty(M * H, 64, device=dev, dtype=torch.bfloat16)
    nv.gemm(qn, wg, gate_out, epi=nv.EPI_BIAS_SIGMOID_BF16, colscale=bg)
    torch.cuda.synchronize()
    print("rgpt_b200.prof: ok")


def bandwidth_and_optimizer() -> None:
    from rgpt_b200.optimizer import Muon, newton_schulz_batched_f32, _NSWorkspaceF32

    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(1)
    def rb(*shape):
        return torch.randn(*shape, device=dev, generator=g).bfloat16()
    def rf(*shape):
        return torch.randn(*shape, device=dev, generator=g)

    B, T, H, d, V = 16, 1024, 8, 512, 50304
    M = B * T
    # rownorm forward (RMSNorm, (1 + w)) and backward with the residual-gradient add and dw
    x, w = rf(M, d), rf(d) * 0.1
    y = torch.empty(M, d, device=dev, dtype=torch.bfloat16)
    nv.rownorm_fwd(x, y, nv.NORM_RMS_AFFINE, 1e-5, w=w)
    dy, gi = rf(M, d), rf(M, d)
    go = torch.empty(M, d, device=dev); gb = torch.empty(M, d, device=dev, dtype=torch.bfloat16)
    dw = torch.zeros(d, device=dev)
    nv.rownorm_bwd(x, dy, nv.NORM_RMS_AFFINE, 1e-5, go, w=w, g_in=gi, g_bf16=gb, dw=dw)
    # QKV prep (f_rmsnorm QK norm, RoPE, normalised q for the G1 gate) forward and backward
    qkv = rb(M, 3 * d)
    qk = torch.empty(M, 2 * d, device=dev, dtype=torch.bfloat16); qn = torch.empty(M, d, device=dev,
                                                                                     dtype=torch.bfloat16)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=dev, dtype=torch.float32) / 64))
    nv.qkv_prep_fwd(qkv, qk, qn, inv_freq, nv.NORM_RMS, nv.FLT_EPS, 0.5, M, T, H)
    dq, dk, dqn, dgp = rf(M, d), rf(M, d), rf(M, d), rb(M, d)
    dqkv = torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16); dbg = torch.zeros(64, device=dev)
    nv.qkv_prep_bwd(qkv, dq, dk, dqn, dgp, dqkv, inv_freq, nv.NORM_RMS, nv.FLT_EPS, 0.5, M, T, H, dbg=dbg)
    # attention backward prep (gate product, D = rowsum(do * o), dq zeroing)
    dog, o = rb(M, d), rb(M, d)
    gate = torch.sigmoid(rf(M, d)).bfloat16()
    do, dgate = torch.empty_like(o), torch.empty_like(o)
    D = torch.empty(B, H, T, device=dev)
    nv.attn_bwd_prep(dog, o, gate, do, dgate, D, B, T, H, dq_zero=dq)
    del qkv, qk, qn, dqkv, dk, dqn, dgp, dog, do, dgate
    # embedding forward / backward
    ids = torch.randint(0, V, (M,), device=dev, generator=g)
    emb = rf(V, d) * 0.02
    xe = torch.empty(M, d, device=dev)
    nv.embedding_fwd(ids, emb, xe)
    demb = torch.zeros(V, d, device=dev)
    nv.embedding_bwd(ids, dy, demb)
    del emb, demb, xe
    # cross entropy over the whole step's logits, gradient in place
    logits = rb(M, V)
    labels = torch.randint(0, V, (M,), device=dev, generator=g)
    rows = torch.empty(M, device=dev); sb = torch.empty(4, device=dev); lo = torch.empty(1, device=dev)
    nv.cross_entropy(logits, labels, loss_rows=rows, scale_buf=sb, loss_out=lo, write_grad=True)
    del logits
    torch.cuda.synchronize(); torch.cuda.empty_cache()
    # one optimizer step over the gpt-small parameter shapes (the Trainer's groups)
    L = 8
    mats = [torch.nn.Parameter(rf(*s) * 0.02) for _ in range(L)
            for s in [(d, d)] * 4 + [(4 * d, d), (d, 4 * d), (64, 64)]]
    big = [torch.nn.Parameter(rf(V, d) * 0.02), torch.nn.Parameter(rf(V, d) * 0.02)]  # embs, lm_head
    vecs = [torch.nn.Parameter(torch.zeros(d, device=dev)) for _ in range(2 * L + 1)] + \
           [torch.nn.Parameter(torch.zeros(64, device=dev)) for _ in range(L)]
    for p_ in mats + big + vecs:
        p_.grad = torch.randn(p_.shape, device=dev, generator=g) * 1e-3
    opt = Muon([{"params": mats, "use_muon": True}, {"params": big[1:], "use_muon": False, "weight_decay": 0.1},
                {"params": big[:1] + vecs, "use_muon": False, "weight_decay": 0.0}],
               lr=6e-4, weight_decay=0.1, muon_lr_multiplier=33.3)
    opt.step()
    torch.cuda.synchronize()
    del opt, mats, big, vecs; torch.cuda.empty_cache()
    # one fp32 Newton-Schulz iteration of one [512, 2048] matrix (hi/lo split, POLY_F32)
    ws = _NSWorkspaceF32(1, d, 4 * d, dev)
    ws.X.copy_(rf(1, d, 4 * d) * (1.0 / 1024))
    newton_schulz_batched_f32(ws, 1)
    # dropout 0.1: attention forward and the residual GEMM with the branch mask
    qk2, qkv2 = rb(M, 2 * d), rb(M, 3 * d)
    o2, og2 = torch.empty(M, d, device=dev, dtype=torch.bfloat16), torch.empty(M, d, device=dev,
                                                                                  dtype=torch.bfloat16)
    lse = torch.empty(B, H, T, device=dev)
    seed = torch.tensor([12345], dtype=torch.int64, device=dev)
    amask = torch.empty(B * H, T // 32, T, device=dev, dtype=torch.int32)
    adrop = nv.Drop(amask, seed, 2, 0.1)
    nv.attn_drop_mask(adrop, B, T, H)
    nv.attn_fwd(qk2, qkv2, gate, o2, og2, lse, B, T, H, drop=adrop)
    wo = rb(d, d)
    hout = torch.empty(M, d, device=dev)
    rmask = torch.empty(M, d // 32, device=dev, dtype=torch.int32)
    rdrop = nv.Drop(rmask, seed, 0, 0.1)
    nv.drop_mask_rows(rdrop, M, d)
    nv.gemm(og2, wo, hout, epi=nv.EPI_RESID_F32, c=x, drop=rdrop)
    torch.cuda.synchronize()
    print("rgpt_b200.prof bw: ok")


def ffn_sweep() -> None:
    """The fused linear+activation sweep: X bf16 [M, 512] ~ N(0, 1), W1 [2048, 512] and W2 [2048, 512]
    ~ N(0, 0.02), no bias, upstream grad ~ N(0, 1), M in {8192, 16384, 32768, 65536}, the four
    activations (model/kernels.py:289-374). Forward = fc1 GEMM with the activation epilogue (pre and
    post stored) + the W2 GEMM; backward = dW2, dpre (activation-gradient epilogue), dW1, dX. Each pass
    is replayed 10 times from a CUDA graph and timed with CUDA events; prints microseconds and TF/s
    over 12 M 512 2048 FLOP (fc1 + act alone: 6 M 512 2048)."""
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(3)
    K, N = 512, 2048
    w1 = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()  # [N, Out], fc2.weight^T
    print("act           M   fwd us   bwd us  total TF/s  (fc1+act fwd us, TF/s)")
    for M in (8192, 16384, 32768, 65536):
        x = torch.randn(M, K, device=dev, generator=g).bfloat16()
        dy = torch.randn(M, K, device=dev, generator=g).bfloat16()
        pre = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        post, dpre = torch.empty_like(pre), torch.empty_like(pre)
        out = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
        dw1, dw2 = torch.zeros(N, K, device=dev), torch.zeros(N, K, device=dev)
        dx = torch.empty(M, K, device=dev)
        for name in ("squared_relu", "gelu", "silu", "mish"):
            act = nv.act_id(name)

            def fc1():
                nv.gemm(x, w1, pre, epi=nv.EPI_ACT_FWD, act=act, out2=post)

            def fwd():
                fc1()
                nv.gemm(post, w2.t(), out)

            def bwd():
                nv.gemm(post.t(), dy.t(), dw2, epi=nv.EPI_ACCUM_F32, splitk=0)
                nv.gemm(dy, w2, dpre, epi=nv.EPI_ACT_BWD, act=act, c=pre)
                nv.gemm(dpre.t(), x.t(), dw1, epi=nv.EPI_ACCUM_F32, splitk=0)
                nv.gemm(dpre, w1.t(), dx, epi=nv.EPI_STORE_F32)

            def timed(fn, n=10):
                fn()
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    for _ in range(n):
                        fn()
                gr.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                gr.replay()
                e1.record()
                torch.cuda.synchronize()
                return e0.elapsed_time(e1) / n * 1e3

            tf, tb, t1 = timed(fwd), timed(bwd), timed(fc1)
            flops = 12.0 * M * K * N
            print(f"{name:12s} {M:6d} {tf:8.1f} {tb:8.1f} {flops / ((tf + tb) * 1e-6) / 1e12:11.1f}"
                  f"  ({t1:.1f}, {2.0 * M * K * N / (t1 * 1e-6) / 1e12:.1f})")
        del x, dy, pre, post, dpre, out, dx
        torch.cuda.empty_cache()


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "bw":
        bandwidth_and_optimizer()
    elif len(sys.argv) > 1 and sys.argv[1] == "ffn":
        ffn_sweep()
    else:
        main()
