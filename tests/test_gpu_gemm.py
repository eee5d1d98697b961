"""tcgen05 GEMM (rgpt_gemm_bf16) against a plain PyTorch fp32 reference.

Tolerance: inputs are bf16, accumulation fp32, so the only differences vs the
fp32 reference of the same bf16 inputs are summation order and the final bf16
rounding of bf16 outputs: rel. Frobenius error <= 1e-2 for bf16 outputs and
<= 1e-4 for fp32 outputs.
"""
import pytest
import torch

from rgpt_b200 import native as nv

pytestmark = pytest.mark.gpu


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def ref_act(name, x):
    import torch.nn.functional as F
    if name == "squared_relu":
        return torch.relu(x) ** 2
    if name == "gelu":
        return F.gelu(x, approximate="tanh")
    if name == "silu":
        return F.silu(x)
    if name == "mish":
        return F.mish(x)
    return x


def ref_act_grad(name, x):
    x = x.detach().clone().requires_grad_(True)
    y = ref_act(name, x)
    (g,) = torch.autograd.grad(y.sum(), x)
    return g


@pytest.mark.parametrize("M,N,K", [(256, 384, 320), (296, 392, 200), (128, 128, 64), (1024, 2048, 512)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_layouts_store_bf16(cuda, M, N, K, a_mn, b_mn):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    A = a.t().contiguous().t() if a_mn else a  # same values, MN-major storage
    B = b.t().contiguous().t() if b_mn else b
    out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    nv.gemm(A, B, out)
    ref = a.float() @ b.float().t()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)])
def test_gemm_store_f32_exactish(cuda, a_mn, b_mn):
    M, N, K = 384, 256, 448
    g = torch.Generator(device=cuda).manual_seed(1)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    A = a.t().contiguous().t() if a_mn else a
    B = b.t().contiguous().t() if b_mn else b
    out = torch.empty(M, N, device=cuda, dtype=torch.float32)
    nv.gemm(A, B, out, epi=nv.EPI_STORE_F32, alpha=0.5)
    ref = 0.5 * (a.float() @ b.float().t())
    assert rel_err(out, ref) < 1e-4


def test_gemm_weight_grad_splitk_accum(cuda):
    # dW += dY^T X with the contraction over a long token dim (split-K + atomics)
    T, Nout, Kin = 8192, 512, 256
    g = torch.Generator(device=cuda).manual_seed(2)
    dy = torch.randn(T, Nout, device=cuda, generator=g).bfloat16()
    x = torch.randn(T, Kin, device=cuda, generator=g).bfloat16()
    dw = torch.randn(Nout, Kin, device=cuda, generator=g)
    ref = dw + dy.float().t() @ x.float()
    nv.gemm(dy.t(), x.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)
    assert rel_err(dw, ref) < 1e-4


@pytest.mark.parametrize("act", ["squared_relu", "gelu", "silu", "mish"])
def test_gemm_act_fwd_bwd(cuda, act):
    M, N, K = 512, 1024, 256
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    pre = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    post = torch.empty_like(pre)
    nv.gemm(x, w, pre, epi=nv.EPI_ACT_FWD, act=nv.act_id(act), out2=post)
    ref_pre = x.float() @ w.float().t()
    assert rel_err(pre, ref_pre) < 1e-2
    assert rel_err(post, ref_act(act, ref_pre)) < 2e-2
    # backward: dpre = (dY @ W2^T) * act'(pre) with W2 [N, Kout] -> here dY [M, 128], W2 [N, 128]
    dy = torch.randn(M, 128, device=cuda, generator=g).bfloat16()
    w2 = (torch.randn(N, 128, device=cuda, generator=g) * 0.05).bfloat16()
    dpre = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    nv.gemm(dy, w2, dpre, epi=nv.EPI_ACT_BWD, act=nv.act_id(act), c=pre)
    ref = (dy.float() @ w2.float().t()) * ref_act_grad(act, pre.float())
    assert rel_err(dpre, ref) < 2e-2


@pytest.mark.parametrize("shape", [(512, 1024, 256), (16384, 2048, 512), (16384, 2048, 1024)],
                         ids=["tile128", "fc1_tile256", "cta_pair"])
def test_gemm_squared_relu_post_only(cuda, shape):
    # ACT_SQRELU_POST: the forward writes only post = relu(acc)^2 (equal, bit for bit, to the two-output
    # epilogue's post), and the backward forms act'(pre) = 2 sqrt(post) from it, within bf16 rounding of
    # 2 relu(pre). Shapes: 128-wide tiles, the model's fc1 (128 x 256 tiles) and a long-K GEMM on CTA pairs.
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    pre = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    post = torch.empty_like(pre)
    nv.gemm(x, w, pre, epi=nv.EPI_ACT_FWD, act=nv.ACT_SQRELU, out2=post)
    post_only = torch.full_like(pre, 7.0)
    nv.gemm(x, w, post_only, epi=nv.EPI_ACT_FWD, act=nv.ACT_SQRELU_POST)
    assert torch.equal(post_only, post)
    dy = torch.randn(M, 128, device=cuda, generator=g).bfloat16()
    w2 = (torch.randn(N, 128, device=cuda, generator=g) * 0.05).bfloat16()
    d_pre, d_post = torch.empty_like(pre), torch.empty_like(pre)
    nv.gemm(dy, w2, d_pre, epi=nv.EPI_ACT_BWD, act=nv.ACT_SQRELU, c=pre)
    nv.gemm(dy, w2, d_post, epi=nv.EPI_ACT_BWD, act=nv.ACT_SQRELU_POST, c=post_only)
    ref = (dy.float() @ w2.float().t()) * 2.0 * (x.float() @ w.float().t()).clamp_min(0)
    assert rel_err(d_post, ref) < 1e-2
    assert rel_err(d_post, d_pre.float()) < 1e-2


@pytest.mark.parametrize("act", ["squared_relu", "gelu", "silu", "mish"])
def test_gemm_act_epilogue_elementwise_wide_range(cuda, act):
    # Every pre-activation value in [-30, 30] (an identity weight passes A through exactly), so the
    # saturated ends and Mish's x > 20 branch are exercised: post = act(pre) and dpre = act'(pre) per
    # element, against torch's fp32 evaluation, within the bf16 rounding of the stored outputs.
    n = 128
    vals = torch.linspace(-30.0, 30.0, n * n, device=cuda).view(n, n).bfloat16()
    eye = torch.eye(n, device=cuda).bfloat16()
    pre = torch.empty(n, n, device=cuda, dtype=torch.bfloat16)
    post = torch.empty_like(pre)
    nv.gemm(vals, eye, pre, epi=nv.EPI_ACT_FWD, act=nv.act_id(act), out2=post)
    x = vals.float()
    assert torch.equal(pre.float(), x)
    ref = ref_act(act, x)
    assert torch.allclose(post.float(), ref, rtol=1e-2, atol=1e-5), (post.float() - ref).abs().max()
    dpre = torch.empty_like(pre)
    nv.gemm(torch.ones(n, n, device=cuda).bfloat16(), eye, dpre, epi=nv.EPI_ACT_BWD, act=nv.act_id(act), c=pre)
    gref = ref_act_grad(act, x)
    assert torch.allclose(dpre.float(), gref, rtol=1e-2, atol=1e-5), (dpre.float() - gref).abs().max()


def test_gemm_resid_colscale(cuda):
    M, N, K = 1024, 512, 512
    g = torch.Generator(device=cuda).manual_seed(4)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    x = torch.randn(M, N, device=cuda, generator=g)
    ls = torch.rand(N, device=cuda, generator=g)
    ref = x + (a.float() @ w.float().t()) * ls
    out = torch.empty_like(x)
    nv.gemm(a, w, out, epi=nv.EPI_RESID_F32, c=x, colscale=ls)
    assert rel_err(out, ref) < 1e-5
    # in place, no scale
    ref2 = x + a.float() @ w.float().t()
    nv.gemm(a, w, x, epi=nv.EPI_RESID_F32, c=x)
    assert rel_err(x, ref2) < 1e-5


def test_gemm_batched_poly(cuda):
    # X' = a*X + (B @ X) batched, with B symmetric, X MN-major as the B operand
    nb, R, C = 6, 256, 512
    g = torch.Generator(device=cuda).manual_seed(5)
    X = (torch.randn(nb, R, C, device=cuda, generator=g) * 0.05).bfloat16()
    S = torch.randn(nb, R, R, device=cuda, generator=g)
    Bm = ((S + S.transpose(1, 2)) * 0.05).bfloat16()
    out = torch.empty_like(X)
    # logical B operand [N=C, K=R] = X^T per batch -> X.transpose(1,2) has unit stride on N
    nv.gemm(Bm, X.transpose(1, 2), out, epi=nv.EPI_POLY_BF16, alpha=1.0, beta=3.4445, c=X)
    ref = 3.4445 * X.float() + Bm.float() @ X.float()
    assert rel_err(out, ref) < 1e-2
    # A = X X^T batched (both K-major)
    A = torch.empty(nb, R, R, device=cuda, dtype=torch.bfloat16)
    nv.gemm(X, X, A)
    assert rel_err(A, X.float() @ X.float().transpose(1, 2)) < 1e-2


def test_gemm_lm_head_shape(cuda):
    # vocab-sized N (not a multiple of the 256-wide tile)
    M, N, K = 2048, 50304, 512
    g = torch.Generator(device=cuda).manual_seed(6)
    h = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    out = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    nv.gemm(h, w, out)
    assert rel_err(out, h.float() @ w.float().t()) < 1e-2


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True), (False, True)])
def test_gemm_small_and_ragged_shapes(cuda, a_mn, b_mn):
    # the reference kernel test's own shapes (M,N,K,Out = 128,256,128,64) and smaller edges
    for M, N, K in [(128, 64, 256), (40, 24, 72), (64, 200, 8)]:
        g = torch.Generator(device=cuda).manual_seed(M + N + K)
        a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
        b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
        A = a.t().contiguous().t() if a_mn else a
        B = b.t().contiguous().t() if b_mn else b
        out = torch.empty(M, N, device=cuda, dtype=torch.float32)
        nv.gemm(A, B, out, epi=nv.EPI_STORE_F32)
        assert rel_err(out, a.float() @ b.float().t()) < 1e-4, (M, N, K)


def test_gemm_rejects_misaligned_leading_dim(cuda):
    a = torch.randn(128, 100, device=cuda).bfloat16()[:, :99]  # ld 100 -> 200 bytes, not a multiple of 16
    out = torch.empty(128, 128, device=cuda, dtype=torch.bfloat16)
    w = torch.randn(128, 99, device=cuda).bfloat16()
    with pytest.raises(RuntimeError, match="16 bytes"):
        nv.gemm(a, w, out)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_cta_pair_ragged(cuda, a_mn, b_mn):
    # Large enough for the CTA-pair (256 x 256) tiles; M, N and K are not tile multiples, and
    # the last row tile leaves the second CTA of its pair without any valid row.
    M, N, K = 4160, 2104, 1096
    g = torch.Generator(device=cuda).manual_seed(11)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(N, K, device=cuda, generator=g).bfloat16()
    A = a.t().contiguous().t() if a_mn else a
    B = b.t().contiguous().t() if b_mn else b
    ref = a.float() @ b.float().t()
    out = torch.empty(M, N + 8, device=cuda, dtype=torch.bfloat16)[:, :N]  # padded leading dim
    nv.gemm(A, B, out)
    assert rel_err(out, ref) < 1e-2
    out32 = torch.empty(M, N, device=cuda, dtype=torch.float32)
    nv.gemm(A, B, out32, epi=nv.EPI_STORE_F32, alpha=0.25)
    assert rel_err(out32, 0.25 * ref) < 1e-4
    pre = torch.empty(M, N + 8, device=cuda, dtype=torch.bfloat16)[:, :N]
    post = torch.empty(M, N + 8, device=cuda, dtype=torch.bfloat16)[:, :N]
    nv.gemm(A, B, pre, epi=nv.EPI_ACT_FWD, act=nv.act_id("squared_relu"), out2=post)
    assert rel_err(post, torch.relu(ref) ** 2) < 2e-2
    x = torch.randn(M, N, device=cuda, generator=g)
    res = torch.empty_like(x)
    nv.gemm(A, B, res, epi=nv.EPI_RESID_F32, c=x)
    assert rel_err(res, x + ref) < 1e-5


def test_gemm_cta_pair_batched_poly_and_accum(cuda):
    # Newton-Schulz-sized batched product on CTA pairs, and a long-K weight-gradient GEMM
    nb, R, C = 16, 1024, 2048
    g = torch.Generator(device=cuda).manual_seed(12)
    X = (torch.randn(nb, R, C, device=cuda, generator=g) * 0.05).bfloat16()
    S = torch.randn(nb, R, R, device=cuda, generator=g)
    Bm = ((S + S.transpose(1, 2)) * 0.05).bfloat16()
    out = torch.empty_like(X)
    nv.gemm(Bm, X.transpose(1, 2), out, epi=nv.EPI_POLY_BF16, alpha=1.0, beta=-4.775, c=X)
    assert rel_err(out, -4.775 * X.float() + Bm.float() @ X.float()) < 1e-2
    T, Nout, Kin = 16384, 1536, 512
    dy = torch.randn(T, Nout, device=cuda, generator=g).bfloat16()
    xin = torch.randn(T, Kin, device=cuda, generator=g).bfloat16()
    dw = torch.randn(Nout, Kin, device=cuda, generator=g)
    ref = dw + dy.float().t() @ xin.float()
    nv.gemm(dy.t(), xin.t(), dw, epi=nv.EPI_ACCUM_F32, splitk=0)
    assert rel_err(dw, ref) < 1e-4


@pytest.mark.parametrize("M,N,K", [(300, 1003, 200), (4160, 2043, 1096)])
def test_gemm_c_epilogues_ragged_edges(cuda, M, N, K):
    # Epilogues that read an input C (activation backward, residual add, Newton-Schulz polynomial)
    # with ragged M, N not a multiple of the 16-byte vector, and padded leading dimensions; the
    # second shape runs on CTA pairs.
    g = torch.Generator(device=cuda).manual_seed(13)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    ref = a.float() @ w.float().t()
    ldb = (N + 7) // 8 * 8 + 8  # bf16 leading dims: multiples of 8 elements (16 bytes)
    ldf = (N + 3) // 4 * 4 + 4  # fp32 leading dims: multiples of 4
    pre = torch.randn(M, ldb, device=cuda, generator=g).bfloat16()[:, :N]
    dpre = torch.full((M, ldb), 7.0, device=cuda, dtype=torch.bfloat16)[:, :N]
    nv.gemm(a, w, dpre, epi=nv.EPI_ACT_BWD, act=nv.act_id("squared_relu"), c=pre)
    assert rel_err(dpre, ref * ref_act_grad("squared_relu", pre.float())) < 2e-2
    x = torch.randn(M, ldf, device=cuda, generator=g)[:, :N]
    res = torch.full((M, ldf), 7.0, device=cuda)[:, :N]
    nv.gemm(a, w, res, epi=nv.EPI_RESID_F32, c=x)
    assert rel_err(res, x + ref) < 1e-5
    c = torch.randn(M, ldb, device=cuda, generator=g).bfloat16()[:, :N]
    out = torch.full((M, ldb), 7.0, device=cuda, dtype=torch.bfloat16)[:, :N]
    nv.gemm(a, w, out, epi=nv.EPI_POLY_BF16, alpha=0.5, beta=-1.5, c=c)
    assert rel_err(out, 0.5 * ref - 1.5 * c.float()) < 1e-2


@pytest.mark.parametrize("M,N", [(4096, 50304), (333, 1000), (300, 200)])
def test_gemm_argmax_equals_stored_logits_argmax(cuda, M, N):
    # The argmax epilogue (no logits stored) against the stored bf16 logits of the same GEMM, reduced
    # by the cross-entropy kernel's argmax: identical indices (first maximum on ties), including rows
    # with planted exact ties.
    g = torch.Generator(device=cuda).manual_seed(M + N)
    a = torch.randn(M, 512, device=cuda, generator=g).bfloat16()
    b = (torch.randn(N, 512, device=cuda, generator=g) * 0.05).bfloat16()
    b[N // 2] = b[N // 3]  # two equal columns: the first one must win where they are the maximum
    a[0] = b[N // 3]       # row 0 peaks at those two columns
    logits = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    nv.gemm(a, b, logits)
    ref = torch.empty(M, device=cuda, dtype=torch.int32)
    nv.cross_entropy(logits, torch.zeros(M, device=cuda, dtype=torch.long), argmax=ref)
    pv = torch.empty(M, (N + 127) // 128, device=cuda)
    pi = torch.empty(M, (N + 127) // 128, device=cuda, dtype=torch.int32)
    out = torch.empty(M, device=cuda, dtype=torch.int32)
    nv.gemm_argmax(a, b, pv, pi, out)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert torch.equal(out.long(), logits.float().argmax(dim=1).int().long())
    assert out[0].item() == N // 3
