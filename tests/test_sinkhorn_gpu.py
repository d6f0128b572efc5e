"""GPU parity of the batched Sinkhorn-Knopp projection (hc_sinkhorn_fwd/bwd)
against MHC's own method (hyperconnections/mhc.py:97-102, fixtures made with
autograd by tests/golden/make_golden.py) and the float64 oracle. Float32:
forward to 1e-5 relative (1e-6 absolute), gradients to 1e-5 relative to their
largest magnitude."""

import numpy as np
import pytest
import torch

from oracle import sinkhorn as osk
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

SINK = load_golden("sinkhorn.npz")


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def run(H, G, iters):
    from hyperconnections_b200.ops import sinkhorn_knopp

    Hr = H.clone().requires_grad_(True)
    P = sinkhorn_knopp(Hr, iters)
    P.backward(G)
    return P.detach().double().cpu().numpy(), Hr.grad.double().cpu().numpy()


def check(P, dH, refP, refdH):
    np.testing.assert_allclose(P, refP, rtol=1e-5, atol=1e-6)
    assert np.abs(dH - refdH).max() <= 1e-5 * max(1.0, np.abs(refdH).max())


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in SINK}))
def test_matches_reference(case):
    g = lambda name: SINK[f"{case}_{name}"]  # noqa: E731
    iters = int(g("meta")[2])
    P, dH = run(torch.from_numpy(g("H")).cuda(), torch.from_numpy(g("G")).cuda(), iters)
    check(P, dH, g("P"), g("dH"))


@pytest.mark.parametrize("n", range(1, 9))
@pytest.mark.parametrize("iters", [0, 1, 20, 32, 40])  # <= 32: linear-time backward; 40: prefix recompute
def test_matches_oracle(n, iters):
    g = torch.Generator().manual_seed(n * 100 + iters)
    B = 1000  # not a multiple of the 128-matrix CTA
    H = torch.randn(B, n, n, generator=g) + torch.eye(n)
    G = torch.randn(B, n, n, generator=g)
    P, dH = run(H.cuda(), G.cuda(), iters)
    check(P, dH, osk.sinkhorn_fwd(H.numpy(), iters), osk.sinkhorn_bwd(H.numpy(), G.numpy(), iters))


def test_doubly_stochastic_and_shapes():
    from hyperconnections_b200.ops import sinkhorn_knopp

    H = torch.randn(2, 3, 16384 // 6, 4, 4, device="cuda")[:, :, :100]
    P = sinkhorn_knopp(H)
    assert P.shape == H.shape
    np.testing.assert_allclose(P.sum(-2).cpu().numpy(), 1.0, atol=1e-5)
    np.testing.assert_allclose(P.sum(-1).cpu().numpy(), 1.0, atol=1e-3)  # rows converge, columns exact


def test_errors():
    from hyperconnections_b200.ops import sinkhorn_knopp

    with pytest.raises(RuntimeError, match="CUDA"):
        sinkhorn_knopp(torch.randn(2, 4, 4))
    with pytest.raises(RuntimeError, match="n <= 8"):
        sinkhorn_knopp(torch.randn(2, 9, 9, device="cuda"))
    with pytest.raises(RuntimeError, match="iters"):
        sinkhorn_knopp(torch.randn(2, 4, 4, device="cuda"), iters=1000)
