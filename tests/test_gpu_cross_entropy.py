"""Row-wise cross entropy with the in-place bf16 gradient (trainer.py:148, model/gpt.py:119-120)
against torch fp32 on the same bf16 logits.

Both kernels: the shared-memory row kernel (V % 8 == 0, the row fits in shared memory) and the
streaming kernel (any other V; the logits then sit in a buffer whose leading dimension is padded
to 16 bytes, which the entry point requires). Tolerances: per-row losses 1e-5 relative (fp32
sums); argmax exact (first index of the maximum); dlogits within one bf16 ulp of the fp32 gradient
plus 2^-11 of the row's largest softmax value times the scale (the shared-memory kernel keeps
exp(x - max) as fp16 between its passes).
"""
import pytest
import torch

from rgpt_b200 import native as nv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,V", [(64, 50304), (96, 1000), (48, 1001)])
def test_cross_entropy_rows_loss_argmax_and_grad(cuda, M, V):
    g = torch.Generator(device=cuda).manual_seed(M + V)
    ld = (V + 7) // 8 * 8
    store = torch.zeros(M, ld, device=cuda, dtype=torch.bfloat16)
    logits = store[:, :V]
    logits.copy_((torch.randn(M, V, device=cuda, generator=g) * 3.0).bfloat16())
    logits[3, 17] = logits[3].max() + 1.0  # a clear maximum
    logits[5, 9] = logits[5, 700] = 40.0   # a tie: the first index wins
    labels = torch.randint(0, V, (M,), device=cuda, generator=g)
    labels[1] = -100
    labels[2] = -100
    ref_x = logits.float()
    lse = torch.logsumexp(ref_x, dim=1)
    valid = labels != -100
    safe = labels.clamp_min(0)
    ref_rows = torch.where(valid, lse - ref_x.gather(1, safe[:, None])[:, 0], torch.zeros_like(lse))
    count = valid.sum().float()
    grad_scale = 0.75
    sc = grad_scale / count
    p = torch.softmax(ref_x, dim=1)
    onehot = torch.zeros_like(p).scatter_(1, safe[:, None], 1.0)
    ref_grad = torch.where(valid[:, None], (p - onehot) * sc, torch.zeros_like(p))

    rows = torch.empty(M, device=cuda)
    amax = torch.empty(M, device=cuda, dtype=torch.int32)
    sb = torch.empty(4, device=cuda)
    lo = torch.empty(1, device=cuda)
    nv.cross_entropy(logits, labels, grad_scale=grad_scale, loss_rows=rows, argmax=amax, scale_buf=sb, loss_out=lo,
                     write_grad=True)
    torch.cuda.synchronize()
    torch.testing.assert_close(rows, ref_rows, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(lo[0], ref_rows.sum() / count, rtol=1e-5, atol=1e-6)
    ref_amax = torch.argmax(ref_x, dim=1)  # torch returns the first index of the maximum
    assert torch.equal(amax.long(), ref_amax)
    assert amax[5].item() == 9
    got = logits.float()
    ulp = torch.where(ref_grad == 0, torch.zeros_like(ref_grad), 2.0 ** (torch.floor(torch.log2(ref_grad.abs())) - 7))
    tol = ulp + (2.0 ** -11) * p.max(dim=1, keepdim=True).values * sc + 1e-12
    assert ((got - ref_grad).abs() <= tol).all(), (got - ref_grad).abs().max()
    assert (logits[~valid] == 0).all()
    if ld > V:
        assert (store[:, V:] == 0).all()  # the padding past V is untouched
