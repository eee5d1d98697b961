"""The persistent Newton-Schulz chain kernel (rgpt_ns_chain) against the batched-GEMM path and the oracle.

Both paths run the same GEMMs with bf16 operands, fp32 accumulation over the same k order and the same
fused polynomial epilogues, so their results agree to within bf16 rounding of the last step (tolerance
1e-2 relative Frobenius: tile shapes differ, which can change where an fp32 sum of products rounds).
Against the oracle's bf16 restatement of optimizer.py:18-45 (which rounds after every op) the bound is
the 5e-2 of the other Newton-Schulz tests. Shapes cover every shape class of the training step and the
single-matrix Muon step, including a matrix narrower than one 128-wide tile and a batch whose unit
count is far below the SM count, on both tile schemes (single-CTA 128 x 128 tiles and CTA-pair 256 x 256
tiles, the latter also with padded rows and columns).
"""
import pytest
import torch

from oracle import ref_ops as O
from rgpt_b200.optimizer import _NSWorkspace, _pad8, newton_schulz_batched
from rgpt_b200 import native as nv

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _ws(G, dev):
    n, R, C = G.shape
    xr, xc = (C, R) if R > C else (R, C)
    ws = _NSWorkspace(n, xr, xc, dev)
    Xs = G.transpose(1, 2) if R > C else G
    ws.X[:, :xr, :xc].copy_(Xs.to(dev).to(torch.bfloat16))
    ws.sumsq.copy_(ws.X.float().pow(2).sum(dim=(1, 2)))
    nv.ns_scale(ws.X, xr, _pad8(xc), n, ws.sumsq)
    return ws, xr, xc


# CTA-pair tiles: (32, 512, 512), (16, 512, 2048) and the padded (32, 200, 328); single-CTA tiles: the rest
@pytest.mark.parametrize("shape", [(32, 512, 512), (16, 512, 2048), (8, 64, 64), (1, 2048, 512), (3, 200, 328),
                                   (32, 200, 328)])
def test_chain_matches_batched_and_oracle(cuda, shape):
    g = torch.Generator().manual_seed(sum(shape))
    G = torch.randn(*shape, generator=g) * 1e-2
    ws_c, xr, xc = _ws(G, cuda)
    ws_b, _, _ = _ws(G, cuda)
    out_c = newton_schulz_batched(ws_c, 5, impl="chain")[:, :xr, :xc].float()
    out_b = newton_schulz_batched(ws_b, 5, impl="batched")[:, :xr, :xc].float()
    torch.cuda.synchronize()
    assert nv._lib.device_error() == 0
    assert torch.isfinite(out_c).all()
    assert rel(out_c, out_b) < 1e-2, rel(out_c, out_b)
    ref = O.zeropower_ns5(G, 5)  # bf16 restatement, per matrix
    ref = ref.transpose(1, 2) if shape[1] > shape[2] else ref
    assert rel(out_c, ref.float()) < 5e-2, rel(out_c, ref.float())


@pytest.mark.parametrize("n", [4, 32], ids=["single_cta_tiles", "cta_pair_tiles"])
def test_chain_twice_in_a_row_and_padding_untouched(cuda, n):
    """Two calls on the same workspace (the counters are re-zeroed each call); the padded rows/columns
    of the buffers stay zero."""
    G = torch.randn(n, 196, 324, generator=torch.Generator().manual_seed(3)) * 1e-2
    ws, xr, xc = _ws(G, cuda)
    first = newton_schulz_batched(ws, 5, impl="chain").clone()
    ws2, _, _ = _ws(G, cuda)
    ws2.ctr = ws.ctr  # shared counter buffer, as two calls of one optimizer step
    second = newton_schulz_batched(ws2, 5, impl="chain")
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    assert first[:, xr:, :].abs().sum().item() == 0 and first[:, :, xc:].abs().sum().item() == 0
