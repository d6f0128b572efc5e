"""GPU parity of stream_mix_add for 9 <= N <= 32 (the shared-memory kernels,
and the ring kernel on the tensor cores for half-precision streams),
against the reference's small-NB Function run on CPU (tests/golden/
stream_mix_large_n.npz) and the float64 oracle. Tolerances as for N <= 8:
1e-5 relative in fp32; 2e-2 (bf16) / 1e-2 (fp16) absolute wherever |ref| < 8,
half an ulp more where |ref| >= 8 (tests/parity.py), against the oracle of
the same half-precision inputs; parameter gradients 1e-5
relative (fp32 sums over D), or the rounding of Phi's dtype when Phi is half
precision, since they are returned in that dtype."""

import numpy as np
import pytest
import torch

from oracle import stream_mix as omix
from tests.conftest import load_golden
from tests.parity import assert_half

pytestmark = pytest.mark.gpu

MIXL = load_golden("stream_mix_large_n.npz")


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def np64(t):
    return t.detach().double().cpu().numpy()


def rel(got, ref, tol, what):
    got = np64(got) if torch.is_tensor(got) else got
    err = np.abs(got - ref).max() if ref.size else 0.0
    bound = tol * max(1.0, np.abs(ref).max() if ref.size else 0.0)
    assert err <= bound, f"{what}: max err {err:.3e} > {bound:.3e}"


def half(got, ref, what):
    assert_half(got, ref, what)


def run(Phi, x, Y, v, G):
    from hyperconnections_b200.ops import stream_mix_add

    ts = [t.detach().clone().requires_grad_(True) for t in (Phi, x, Y)]
    vt = None if v is None else v.detach().clone().requires_grad_(True)
    out = stream_mix_add(*ts, vt)
    out.backward(G)
    return out, ts[0].grad, ts[1].grad, ts[2].grad, (None if vt is None else vt.grad)


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in MIXL}))
def test_matches_reference(case):
    g = lambda name: torch.from_numpy(MIXL[f"{case}_{name}"]).cuda()  # noqa: E731
    proj = bool(MIXL[f"{case}_meta"][3])
    out, gP, gx, gY, gv = run(g("Phi"), g("x"), g("Y"), g("v") if proj else None, g("Gup"))
    ref = lambda name: MIXL[f"{case}_{name}"].astype(np.float64)  # noqa: E731
    rel(out, ref("out"), 1e-5, "out")
    rel(gP, ref("gPhi"), 1e-5, "grad_Phi")
    rel(gx, ref("gx"), 1e-5, "grad_x")
    assert torch.equal(gY, g("Gup"))
    if proj:
        rel(gv, ref("gv"), 1e-5, "grad_v")


def inputs(B, N, D, dtype, proj, seed, phi_dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    Phi = (torch.randn(B, N, N, generator=g) / N**0.5).to(phi_dtype)
    x = torch.randn(B, N, D, generator=g).to(dtype)
    Y = torch.randn(B, N, D, generator=g).to(dtype)
    v = torch.nn.functional.normalize(torch.randn(B, N, generator=g), dim=-1).to(phi_dtype) if proj else None
    G = torch.randn(B, N, D, generator=g).to(dtype)
    return [None if t is None else t.cuda() for t in (Phi, x, Y, v, G)]


def check(Phi, x, Y, v, G, half_streams):
    out, gP, gx, _, gv = run(Phi, x, Y, v, G)
    vs = None if v is None else np64(v)
    ro = omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y), vs)
    rP, rx, _, rv = omix.stream_mix_bwd(np64(G), np64(Phi), np64(x), vs)
    if half_streams:
        half(out, ro, "out")
        half(gx, rx, "grad_x")
    else:
        rel(out, ro, 1e-5, "out")
        rel(gx, rx, 1e-5, "grad_x")
    # parameter gradients come back in Phi's / v's dtype (computed in fp32)
    ptol = 1e-5 if Phi.dtype == torch.float32 else 2.0**-7
    rel(gP, rP, ptol, "grad_Phi")
    if v is not None:
        rel(gv, rv, ptol, "grad_v")


@pytest.mark.parametrize("N", [9, 12, 16, 17, 24, 32])
@pytest.mark.parametrize("proj", [False, True])
@pytest.mark.parametrize("D", [1, 7, 64, 513, 1536])
def test_fp32(N, proj, D):
    check(*inputs(5, N, D, torch.float32, proj, seed=N * 7 + D), half_streams=False)


@pytest.mark.parametrize("N", [12, 16, 32])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("phi_dtype", ["f32", "stream"])
def test_half(N, dtype, phi_dtype):
    pd = torch.float32 if phi_dtype == "f32" else dtype
    check(*inputs(6, N, 1024, dtype, True, seed=N, phi_dtype=pd), half_streams=True)
    check(*inputs(6, N, 1030, dtype, False, seed=N + 1, phi_dtype=pd), half_streams=True)


@pytest.mark.parametrize("N", [9, 17, 24, 32])
@pytest.mark.parametrize("D", [64, 192, 1536])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_ring(N, D, dtype):
    """Half-precision streams with D a multiple of 64: the ring kernel with
    grad_x and the Gram on the tensor cores (whole tokens and slices, Phi in
    fp32 and in the stream dtype, with and without the projection)."""
    check(*inputs(40, N, D, dtype, N % 2 == 1, seed=N * 31 + D), half_streams=True)
    check(*inputs(40, N, D, dtype, N % 2 == 0, seed=N * 37 + D, phi_dtype=dtype), half_streams=True)


def test_half_ring_many_tokens():
    """Many tokens per CTA: every consumer cycles the ring many times."""
    from hyperconnections_b200 import _lib

    for _ in range(2):
        check(*inputs(900, 24, 640, torch.bfloat16, True, seed=5), half_streams=True)
    assert _lib.wait_timeouts() == 0


def test_odd_alignment_views():
    """Rows that are not 32-bit aligned take the element-wise path."""
    Phi, x, Y, v, G = inputs(3, 16, 65, torch.bfloat16, True, seed=3)
    check(Phi, x[..., :64].contiguous()[..., :63].contiguous(), Y[..., :63].contiguous(), v,
          G[..., :63].contiguous(), half_streams=True)


def test_many_tokens_and_grad_subsets():
    from hyperconnections_b200.ops import stream_mix_add

    Phi, x, Y, v, G = inputs(700, 16, 256, torch.bfloat16, True, seed=9)
    X = x.clone().requires_grad_(True)  # only x needs a gradient
    out = stream_mix_add(Phi, X, Y, v)
    out.backward(G)
    rx = omix.stream_mix_bwd(np64(G), np64(Phi), np64(x), np64(v))[1]
    half(X.grad, rx, "grad_x only")


def test_zero_width_gives_zero_parameter_gradients():
    from hyperconnections_b200.ops import stream_mix_add

    Phi = torch.randn(4, 20, 20, device="cuda", requires_grad=True)
    x = torch.empty(4, 20, 0, device="cuda", requires_grad=True)
    out = stream_mix_add(Phi, x, torch.empty(4, 20, 0, device="cuda"))
    out.backward(torch.empty_like(out))
    assert torch.count_nonzero(Phi.grad) == 0
