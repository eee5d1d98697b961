"""rgpt_cross_entropy_noalloc: the cross-entropy entry point for callers that cannot allocate.

Some hosts cannot give this library scratch memory: plugin-style runtimes whose
enqueue contract provides only the input/output buffers, or processes whose device
memory is fully reserved by another framework's allocator. For them the library
keeps the cross-entropy scratch (per-row losses, scale and count) in a static device
array. This test calls both entry points through the C ABI on the same inputs, two
calls in a row with different logits, and requires identical results (same kernels,
same arithmetic: loss bitwise equal, dlogits and argmax equal). It lives in its own
file, collected last, and needs nothing from the other tests.
"""
import pytest
import torch

from rgpt_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_ROWS = 262144


def _call_alloc(logits, labels, grad_scale, write_grad):
    M, V = logits.shape
    dev = logits.device
    loss_rows = torch.empty(M, device=dev, dtype=torch.float32)
    scale_buf = torch.empty(2, device=dev, dtype=torch.float32)
    loss = torch.empty(1, device=dev, dtype=torch.float32)
    amax = torch.empty(M, device=dev, dtype=torch.int32)
    _lib.call("rgpt_cross_entropy", logits.data_ptr(), logits.stride(0), M, V, labels.data_ptr(), -100,
              float(grad_scale), loss_rows.data_ptr(), amax.data_ptr(), scale_buf.data_ptr(), loss.data_ptr(),
              int(write_grad), torch.cuda.current_stream().cuda_stream)
    return loss, amax


def _call_noalloc(logits, labels, grad_scale, write_grad):
    M, V = logits.shape
    loss = torch.empty(1, device=logits.device, dtype=torch.float32)
    amax = torch.empty(M, device=logits.device, dtype=torch.int32)
    _lib.call("rgpt_cross_entropy_noalloc", logits.data_ptr(), logits.stride(0), M, V, labels.data_ptr(), -100,
              float(grad_scale), loss.data_ptr(), amax.data_ptr(), int(write_grad),
              torch.cuda.current_stream().cuda_stream)
    return loss, amax


def test_noalloc_cross_entropy_matches_allocating_entry_point():
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    # calls in a row: a smaller M after a larger one (stale per-row losses of the first call must not
    # reach the second's mean), and a vocabulary that is not a multiple of 8 (the streaming kernel
    # instead of the row-in-shared-memory one; the rows keep a 16-byte-aligned stride)
    cases = [(4096, 50304, 50304, 1.0), (1000, 50304, 50304, 0.25), (3000, 50257, 50264, 0.5)]
    for call, (M, V, ld, scale) in enumerate(cases):
        buf = (torch.randn(M, ld, device=dev, generator=g) * (2.0 + call)).to(torch.bfloat16)
        logits = buf[:, :V]
        labels = torch.randint(0, V, (M,), device=dev, generator=g)
        labels[:: 7 + call] = -100  # ignored positions change the valid count between calls
        a, b = buf.clone(), buf.clone()
        loss_a, amax_a = _call_alloc(a[:, :V], labels, scale, True)
        loss_b, amax_b = _call_noalloc(b[:, :V], labels, scale, True)
        torch.cuda.synchronize()
        assert torch.equal(loss_a, loss_b), (call, loss_a.item(), loss_b.item())
        assert torch.equal(amax_a, amax_b)
        assert torch.equal(a, b)  # in-place dlogits
        ref = torch.nn.functional.cross_entropy(logits.float(), labels, ignore_index=-100)
        assert abs(loss_b.item() - ref.item()) / ref.item() < 1e-3


def test_noalloc_cross_entropy_rejects_too_many_rows():
    dev = torch.device("cuda", 0)
    logits = torch.zeros(MAX_ROWS + 1, 8, device=dev, dtype=torch.bfloat16)
    labels = torch.zeros(MAX_ROWS + 1, device=dev, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="262144 rows"):
        _call_noalloc(logits, labels, 1.0, False)
