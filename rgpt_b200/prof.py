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
"""
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


if __name__ == "__main__":
    main()
