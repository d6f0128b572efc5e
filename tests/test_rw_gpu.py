"""GPU parity tests of the m-block width-read and mix + depth-write
(hc_read_fwd/bwd, hc_mix_write_fwd/bwd through hyperconnections_b200.ops).

Expected values: golden fixtures made by the reference's own composition
(einops read einsum cghc.py:410 -> write einsum :417 -> stream_mix_add :449,
float32 on bf16-exact inputs), and the float64 CPU oracle (oracle.rw) on the
same inputs. Tolerances: 1e-5 relative to the largest magnitude in fp32; in
bf16 / fp16, 2e-2 / 1e-2 absolute wherever |ref| < 8 against the oracle of
the same half-precision inputs, half an ulp more where |ref| >= 8
(tests/parity.py). Parameter gradients (fp32 sums over D) are held to 1e-5
relative.
"""

import numpy as np
import pytest
import torch

from oracle import rw as orw
from tests.conftest import load_golden
from tests.parity import assert_half

pytestmark = pytest.mark.gpu

DEVICE = "cuda"
RW = load_golden("rw.npz")
RW_CASES = sorted({k.split("_")[0] for k in RW})


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def ops():
    from hyperconnections_b200 import ops as o

    return o


def np64(t):
    return t.detach().double().cpu().numpy()


def close(got, ref, what, tol, rel=True):
    dtype = got.dtype if torch.is_tensor(got) else None
    got = np64(got) if torch.is_tensor(got) else got
    if rel:
        err = np.abs(got - ref).max() if ref.size else 0.0
        bound = tol * max(1.0, np.abs(ref).max() if ref.size else 0.0)
        assert err <= bound, f"{what}: max err {err:.3e} > {bound:.3e}"
    else:  # half precision: the absolute bar of its dtype (tol unused)
        assert_half(got, ref, what, dtype=dtype)


def inputs(T, n, m, D, dtype, proj, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, n, D, generator=g).to(dtype)
    f = torch.randn(T, m, D, generator=g).to(dtype)
    R = torch.sigmoid(torch.randn(T, m, n, generator=g))
    W = 2 * torch.sigmoid(torch.randn(T, n, m, generator=g))
    S = torch.triu(0.5 * torch.randn(T, n, n, generator=g), 1)
    H = torch.linalg.matrix_exp(S - S.mT)
    v = torch.nn.functional.normalize(torch.randn(T, n, generator=g), dim=-1) if proj else None
    g_u = torch.randn(T, m, D, generator=g).to(dtype)
    g_x = torch.randn(T, n, D, generator=g).to(dtype)
    dev = lambda t: None if t is None else t.to(DEVICE)  # noqa: E731
    return [dev(t) for t in (x, f, R, W, H, v, g_u, g_x)]


def run_read(R, x, g_u):
    Rr, X = (t.detach().clone().requires_grad_(True) for t in (R, x))
    u = ops().hc_read(Rr, X)
    u.backward(g_u)
    return u, Rr.grad, X.grad


def run_mix_write(H, x, W, f, v, g_x):
    Hr, X, Wr, Fv = (t.detach().clone().requires_grad_(True) for t in (H, x, W, f))
    Vr = None if v is None else v.detach().clone().requires_grad_(True)
    out = ops().hc_mix_write(Hr, X, Wr, Fv, Vr)
    out.backward(g_x)
    return out, Hr.grad, X.grad, Wr.grad, Fv.grad, (None if v is None else Vr.grad)


def check_all(x, f, R, W, H, v, g_u, g_x, stream_tol, rel):
    xs, fs, Rs, Ws, Hs, gus, gxs = (np64(t) for t in (x, f, R, W, H, g_u, g_x))
    vs = None if v is None else np64(v)
    u, gR, gx_r = run_read(R, x, g_u)
    close(u, orw.read_fwd(Rs, xs), "u", stream_tol, rel)
    rgR, rgx_r = orw.read_bwd(gus, Rs, xs)
    close(gx_r, rgx_r, "read grad_x", stream_tol, rel)
    close(gR, rgR, "grad_R", 1e-5)
    out, gH, gx_m, gW, gf, gv = run_mix_write(H, x, W, f, v, g_x)
    close(out, orw.mix_write_fwd(Hs, xs, Ws, fs, vs), "x_out", stream_tol, rel)
    rgH, rgx_m, rgW, rgf, rgv = orw.mix_write_bwd(gxs, Hs, xs, Ws, fs, vs)
    close(gx_m, rgx_m, "mix grad_x", stream_tol, rel)
    close(gf, rgf, "grad_f", stream_tol, rel)
    close(gH, rgH, "grad_H", 1e-5)
    close(gW, rgW, "grad_W", 1e-5)
    if v is not None:
        close(gv, rgv, "grad_v", 1e-5)


# ------------------------------------------------------------ reference golden
@pytest.mark.parametrize("case", RW_CASES)
def test_matches_reference_composition(case):
    g = lambda name: torch.from_numpy(RW[f"{case}_{name}"]).to(DEVICE)  # noqa: E731
    proj = bool(RW[f"{case}_meta"][4])
    v = g("v") if proj else None
    u, gR, gx_r = run_read(g("R"), g("x"), g("g_u"))
    out, gH, gx_m, gW, gf, gv = run_mix_write(g("H"), g("x"), g("W"), g("f"), v, g("g_x"))
    ref = lambda name: RW[f"{case}_{name}"].astype(np.float64)  # noqa: E731
    close(u, ref("u"), "u", 1e-5)
    close(out, ref("x_out"), "x_out", 1e-5)
    close(np64(gx_r) + np64(gx_m), ref("grad_x"), "grad_x", 1e-5)
    close(gf, ref("grad_f"), "grad_f", 1e-5)
    close(gR, ref("grad_R"), "grad_R", 1e-5)
    close(gW, ref("grad_W"), "grad_W", 1e-5)
    close(gH, ref("grad_H"), "grad_H", 1e-5)
    if proj:
        close(gv, ref("grad_v"), "grad_v", 1e-5)


# --------------------------------------------------------------- oracle sweeps
NM = [(n, m) for n in range(1, 9) for m in range(1, 5) if m <= n]


@pytest.mark.parametrize("n,m", NM)
@pytest.mark.parametrize("proj", [False, True])
def test_ring_fp32(n, m, proj):
    check_all(*inputs(300, n, m, 256, torch.float32, proj, seed=n * 10 + m), 1e-5, True)


@pytest.mark.parametrize("n,m", NM)
def test_ring_bf16(n, m):
    check_all(*inputs(300, n, m, 768, torch.bfloat16, n % 2 == 0, seed=100 + n * 10 + m), 2e-2, False)


@pytest.mark.parametrize("n,m,D", [(4, 1, 768), (4, 2, 1024), (2, 1, 64), (3, 3, 16), (8, 4, 128)])
def test_ring_fp16(n, m, D):
    check_all(*inputs(200, n, m, D, torch.float16, True, seed=7), 2e-2, False)


@pytest.mark.parametrize("n,m,D", [(2, 1, 8), (4, 1, 32), (4, 2, 64), (6, 3, 24)])
def test_many_small_tokens_per_cta(n, m, D):
    """Small tokens share ring stages (several tokens per item) and every
    consumer cycles the ring many times."""
    check_all(*inputs(5000, n, m, D, torch.bfloat16, True, seed=11), 2e-2, False)


@pytest.mark.parametrize("n,m,D", [(4, 1, 4096), (4, 2, 6144), (8, 1, 2048), (3, 2, 8192)])
def test_sliced_tokens(n, m, D):
    """Tokens larger than one ring stage are cut into slices."""
    check_all(*inputs(64, n, m, D, torch.bfloat16, n == 4, seed=13), 2e-2, False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,m,D,proj", [(5, 1, 2048, True), (5, 4, 1800, False), (6, 3, 1024, True),
                                        (7, 2, 1536, True), (8, 4, 1024, False), (8, 4, 1800, True),
                                        (8, 2, 2048, True)])
def test_mix_write_sliced_gram(dtype, n, m, D, proj):
    """Half-precision tokens cut into slices at n >= 5: the mix-write
    backward takes its Gram on the tensor cores, on swizzled TMA stages (even
    n, D a multiple of 64) or 16-byte padded rows copied row by row (odd n,
    D = 1800, whose last slice is not a multiple of 16 elements)."""
    check_all(*inputs(150, n, m, D, dtype, proj, seed=17 * n + m + D), 2e-2, False)


@pytest.mark.parametrize("n,m,D", [(2, 1, 1), (4, 2, 7), (4, 4, 2), (6, 3, 33), (3, 1, 100), (2, 4, 16)])
def test_element_wise_path(n, m, D):
    """Odd or tiny block sizes, and m > n, run the element-wise kernels."""
    check_all(*inputs(40, n, m, D, torch.float32, True, seed=17), 1e-5, True)
    check_all(*inputs(40, n, m, D, torch.bfloat16, False, seed=19), 2e-2, False)


def test_unaligned_streams_use_element_wise_path():
    x, f, R, W, H, v, g_u, g_x = inputs(50, 4, 2, 64 + 8, torch.bfloat16, True, seed=23)
    # views whose base is 2 bytes past a 16-byte boundary
    xs = x[..., 1:65].contiguous()[..., :64]
    big = torch.zeros(50 * 4 * 64 + 1, dtype=torch.bfloat16, device=DEVICE)
    xu = big[1:].view(50, 4, 64)
    xu.copy_(xs)
    assert xu.data_ptr() % 16 != 0
    u = ops().hc_read(R, xu)
    close(u, orw.read_fwd(np64(R), np64(xs)), "u (unaligned)", 2e-2, False)


def test_broadcast_projection_direction():
    """projection='mean' passes one direction [1, n] for every token
    (cghc.py:341-343); its gradient is the sum over the tokens."""
    T, n, m, D = 30, 4, 2, 64
    x, f, R, W, H, _, g_u, g_x = inputs(T, n, m, D, torch.float32, False, seed=29)
    v1 = torch.full((1, n), n ** -0.5, device=DEVICE, requires_grad=True)
    out = ops().hc_mix_write(H, x, W, f, v1)
    out.backward(g_x)
    vs = np.repeat(np64(v1), T, axis=0)
    close(out, orw.mix_write_fwd(np64(H), np64(x), np64(W), np64(f), vs), "x_out", 1e-5)
    rgv = orw.mix_write_bwd(np64(g_x), np64(H), np64(x), np64(W), np64(f), vs)[4]
    assert v1.grad.shape == (1, n)
    close(v1.grad, rgv.sum(0, keepdims=True), "grad_v", 1e-5)


def test_leading_dims_and_needs_input_grad():
    B, S, n, m, D = 2, 5, 4, 2, 64
    x, f, R, W, H, v, g_u, g_x = inputs(B * S, n, m, D, torch.float32, True, seed=31)
    shape = lambda t, *s: t.view(B, S, *s)  # noqa: E731
    X = shape(x, n, D).clone().requires_grad_(True)
    out = ops().hc_mix_write(shape(H, n, n), X, shape(W, n, m), shape(f, m, D), shape(v, n))
    assert out.shape == (B, S, n, D)
    out.backward(shape(g_x, n, D))
    rgx = orw.mix_write_bwd(np64(g_x), np64(H), np64(x), np64(W), np64(f), np64(v))[1]
    close(X.grad.view(B * S, n, D), rgx, "grad_x only", 1e-5)
    Rr = shape(R, m, n).clone().requires_grad_(True)
    u = ops().hc_read(Rr, shape(x, n, D))
    u.backward(shape(g_u, m, D))
    close(Rr.grad.view(B * S, m, n), orw.read_bwd(np64(g_u), np64(R), np64(x))[0], "grad_R only", 1e-5)


def test_m1_matches_fused_step():
    """With m = 1 the read and the mix-write are the two halves of the fused
    step (R = alpha, W = beta)."""
    T, n, D = 500, 4, 768
    g = torch.Generator().manual_seed(37)
    x = torch.randn(T, n, D, generator=g).to(torch.bfloat16).to(DEVICE)
    f = torch.randn(T, D, generator=g).to(torch.bfloat16).to(DEVICE)
    S = torch.triu(0.5 * torch.randn(T, n, n, generator=g), 1)
    H = torch.linalg.matrix_exp(S - S.mT).to(DEVICE)
    alpha = torch.softmax(torch.randn(T, n, generator=g), -1).to(DEVICE)
    beta = torch.softmax(torch.randn(T, n, generator=g), -1).to(DEVICE)
    u_f, x_f = ops().stream_mix_fused(x, f, H, alpha, beta)
    u_r = ops().hc_read(alpha[:, None, :], x)[:, 0]
    x_r = ops().hc_mix_write(H, x, beta[:, :, None], f[:, None, :])
    # same fp32 terms in the same order; at most one bf16 rounding step apart
    assert (u_f.float() - u_r.float()).abs().max().item() <= 2.0**-7 * max(1.0, u_f.float().abs().max().item())
    assert (x_f.float() - x_r.float()).abs().max().item() <= 2.0**-7 * max(1.0, x_f.float().abs().max().item())


def test_zero_block_size_gives_zero_parameter_gradients():
    T, n, m = 6, 3, 2
    x = torch.empty(T, n, 0, device=DEVICE, requires_grad=True)
    f = torch.empty(T, m, 0, device=DEVICE, requires_grad=True)
    H = torch.eye(n, device=DEVICE).expand(T, n, n).contiguous().requires_grad_(True)
    W = torch.ones(T, n, m, device=DEVICE, requires_grad=True)
    out = ops().hc_mix_write(H, x, W, f)
    out.backward(torch.empty_like(out))
    assert torch.count_nonzero(H.grad) == 0 and torch.count_nonzero(W.grad) == 0


def test_errors():
    o = ops()
    x = torch.randn(4, 2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        o.hc_read(torch.rand(4, 1, 2), x)
    xc = x.to(DEVICE)
    with pytest.raises(RuntimeError, match="m <= 4"):
        o.hc_read(torch.rand(4, 5, 2, device=DEVICE), xc)
    with pytest.raises(RuntimeError, match="n <= 8"):
        o.hc_mix_write(torch.rand(4, 9, 9, device=DEVICE), torch.randn(4, 9, 8, device=DEVICE),
                       torch.rand(4, 9, 1, device=DEVICE), torch.randn(4, 1, 8, device=DEVICE))
    with pytest.raises(AssertionError):
        o.hc_mix_write(torch.rand(4, 2, 2, device=DEVICE), xc, torch.rand(4, 2, 1, device=DEVICE),
                       torch.randn(4, 2, 8, device=DEVICE))


def test_no_wait_timeouts():
    from hyperconnections_b200 import _lib

    assert _lib.wait_timeouts() == 0
