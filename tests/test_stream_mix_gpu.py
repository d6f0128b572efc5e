"""GPU parity tests of stream_mix_add (hc_stream_mix_fwd / hc_stream_mix_bwd).

Mirrors the reference's tests/test_ops.py (shapes, dtypes, forward, backward,
projection, identity Phi, odd D, N=1, CPU raises) with the CPU oracle
(oracle.stream_mix) as the expected value, plus the golden fixtures made by
the reference's own Triton kernels. Tolerances: the reference's own (1e-4
fp32, 1e-2 fp16) and the tighter parity bar of 1e-5 relative (fp32) / 2e-2
absolute (bf16) / 1e-2 absolute (fp16) wherever |ref| < 8, half an ulp more
where |ref| >= 8 (tests/parity.py).
"""

import numpy as np
import pytest
import torch

from oracle import stream_mix as omix
from tests.conftest import load_golden
from tests.parity import assert_half as _assert_half

pytestmark = pytest.mark.gpu

DEVICE = "cuda"


def _require_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


@pytest.fixture(autouse=True)
def _cuda():
    _require_cuda()


def stream_mix_add(*a, **k):
    from hyperconnections_b200.ops import stream_mix_add as f

    return f(*a, **k)


def make_inputs(B, N, D, dtype=torch.float32, seed=0):
    """Same draws as the reference tests (tests/test_ops.py:48-57), on CPU."""
    torch.manual_seed(seed)
    Phi = torch.randn(B, N, N, dtype=dtype)
    x = torch.randn(B, N, D, dtype=dtype)
    Y = torch.randn(B, N, D, dtype=dtype)
    return Phi.to(DEVICE), x.to(DEVICE), Y.to(DEVICE)


def make_v(B, N, dtype=torch.float32, seed=7):
    torch.manual_seed(seed)
    return torch.nn.functional.normalize(torch.randn(B, N, dtype=dtype), dim=-1).to(DEVICE)


def np64(t):
    return None if t is None else t.detach().double().cpu().numpy()


def assert_half(got, ref, what=""):
    """Half-precision outputs (fp32 accumulation, one rounding to the output
    type): 2e-2 (bf16) / 1e-2 (fp16) absolute where |ref| < 8."""
    _assert_half(got, ref, what)


def assert_rel(got, ref, tol, what=""):
    got = np64(got) if isinstance(got, torch.Tensor) else got
    err = np.abs(got - ref).max() if ref.size else 0.0
    scale = max(np.abs(ref).max() if ref.size else 0.0, 1.0)
    assert err <= tol * scale, f"{what}: max err {err:.3e} > {tol:.1e} * {scale:.3e}"


class TestShapes:
    @pytest.mark.parametrize("B,N,D", [(2, 4, 64), (1, 8, 128), (4, 2, 32)])
    def test_no_proj_shape(self, B, N, D):
        Phi, x, Y = make_inputs(B, N, D)
        assert stream_mix_add(Phi, x, Y).shape == (B, N, D)

    @pytest.mark.parametrize("B,N,D", [(2, 4, 64), (1, 8, 128)])
    def test_proj_shape(self, B, N, D):
        Phi, x, Y = make_inputs(B, N, D)
        assert stream_mix_add(Phi, x, Y, v=make_v(B, N)).shape == (B, N, D)

    @pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
    def test_output_dtype_preserved(self, dtype):
        Phi, x, Y = make_inputs(2, 4, 64, dtype=dtype)
        assert stream_mix_add(Phi, x, Y).dtype == dtype


class TestForward:
    @pytest.mark.parametrize("B,N,D", [(1, 4, 64), (2, 8, 128), (4, 4, 256), (3, 6, 48), (5, 3, 40),
                                       (2, 5, 96), (2, 7, 24), (3, 2, 512), (2, 1, 8)])
    def test_no_proj_fp32(self, B, N, D):
        Phi, x, Y = make_inputs(B, N, D)
        got = stream_mix_add(Phi, x, Y)
        ref = omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y))
        assert torch.allclose(got.double().cpu(), torch.from_numpy(ref), atol=1e-4, rtol=1e-4)
        assert_rel(got, ref, 1e-5, "out")

    @pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
    @pytest.mark.parametrize("B,N,D", [(2, 4, 128), (1, 8, 64), (3, 3, 48)])
    def test_no_proj_half(self, B, N, D, dtype):
        Phi, x, Y = make_inputs(B, N, D, dtype=dtype)
        got = stream_mix_add(Phi, x, Y)
        ref = omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y))
        assert_half(got, ref, "out")

    @pytest.mark.parametrize("B,N,D", [(1, 4, 64), (2, 8, 128), (3, 4, 48), (2, 3, 40), (2, 6, 72)])
    def test_proj_fp32(self, B, N, D):
        Phi, x, Y = make_inputs(B, N, D)
        v = make_v(B, N)
        got = stream_mix_add(Phi, x, Y, v=v)
        ref = omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y), np64(v))
        assert_rel(got, ref, 1e-5, "out(proj)")

    def test_identity_phi_proj_equals_no_proj(self):
        B, N, D = 2, 4, 64
        _, x, Y = make_inputs(B, N, D)
        Phi_id = torch.eye(N, device=DEVICE).unsqueeze(0).expand(B, -1, -1).contiguous()
        v = make_v(B, N)
        assert torch.allclose(stream_mix_add(Phi_id, x, Y, v=v), stream_mix_add(Phi_id, x, Y), atol=1e-5)

    def test_mixed_param_dtypes(self):
        """bf16 streams with fp32 Phi and fp32 v (CGHC "mean" projection)."""
        Phi, x, Y = make_inputs(3, 4, 64)
        xb, Yb = x.bfloat16(), Y.bfloat16()
        v = make_v(3, 4)
        got = stream_mix_add(Phi, xb, Yb, v=v)
        assert got.dtype == torch.bfloat16
        ref = omix.stream_mix_fwd(np64(Phi), np64(xb), np64(Yb), np64(v))
        assert_half(got, ref, "out")

    def test_non_contiguous_and_misaligned_inputs(self):
        """Strided views are made contiguous; an odd element offset takes the
        element-wise path of the same kernel."""
        B, N, D = 3, 4, 64
        Phi, x, Y = make_inputs(B, N, D + 1)
        xs, Ys = x[..., 1:], Y[..., 1:]  # misaligned, non-contiguous
        Phis = torch.randn(B, N, N, device=DEVICE).mT  # transposed view
        got = stream_mix_add(Phis, xs, Ys)
        ref = omix.stream_mix_fwd(np64(Phis), np64(xs), np64(Ys))
        assert_rel(got, ref, 1e-5, "strided")
        flat = torch.randn(B * N * D + 1, device=DEVICE)
        xm = flat[1:].view(B, N, D)  # 4-byte offset: not 16-byte aligned
        got = stream_mix_add(Phi, xm, xm)
        ref = omix.stream_mix_fwd(np64(Phi), np64(xm), np64(xm))
        assert_rel(got, ref, 1e-5, "misaligned")


def _grads(B, N, D, use_proj, dtype=torch.float32, upstream="ones"):
    Phi, x, Y = make_inputs(B, N, D, dtype=dtype)
    v = make_v(B, N, dtype=dtype) if use_proj else None
    Phi_t, x_t, Y_t = (t.detach().requires_grad_(True) for t in (Phi, x, Y))
    v_t = v.detach().requires_grad_(True) if use_proj else None
    out = stream_mix_add(Phi_t, x_t, Y_t, v=v_t)
    if upstream == "ones":
        Gup = torch.ones_like(out)  # .sum().backward() in the reference tests
    else:
        torch.manual_seed(11)
        Gup = torch.randn(out.shape, dtype=out.dtype).to(DEVICE)
    out.backward(Gup)
    ref = omix.stream_mix_bwd(np64(Gup), np64(Phi), np64(x), np64(v))
    return (Phi_t.grad, x_t.grad, Y_t.grad, v_t.grad if use_proj else None), ref, Gup


class TestBackward:
    @pytest.mark.parametrize("upstream", ["ones", "randn"])
    @pytest.mark.parametrize("B,N,D", [(1, 4, 64), (2, 8, 128), (3, 4, 48), (2, 5, 40), (4, 3, 33)])
    def test_grads_no_proj(self, B, N, D, upstream):
        (gP, gx, gY, _), (rP, rx, rY, _), Gup = _grads(B, N, D, False, upstream=upstream)
        assert_rel(gx, rx, 1e-5, "grad_x")
        assert_rel(gP, rP, 1e-5, "grad_Phi")
        assert torch.equal(gY, Gup), "grad_Y must be grad_out itself"
        assert gP.dtype == torch.float32 and gx.dtype == torch.float32

    @pytest.mark.parametrize("upstream", ["ones", "randn"])
    @pytest.mark.parametrize("B,N,D", [(1, 4, 64), (2, 8, 128), (2, 3, 40), (2, 6, 72), (1, 2, 100)])
    def test_grads_proj(self, B, N, D, upstream):
        (gP, gx, gY, gv), (rP, rx, rY, rv), Gup = _grads(B, N, D, True, upstream=upstream)
        assert_rel(gx, rx, 1e-5, "grad_x")
        assert_rel(gP, rP, 1e-5, "grad_Phi")
        assert_rel(gv, rv, 1e-5, "grad_v")

    @pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
    def test_grads_half(self, dtype):
        (gP, gx, _, gv), (rP, rx, _, rv), _ = _grads(3, 4, 96, True, dtype=dtype, upstream="randn")
        assert gP.dtype == dtype and gx.dtype == dtype and gv.dtype == dtype
        assert_half(gx, rx, "grad_x")
        # grad_Phi / grad_v are fp32 sums over D cast to the parameter dtype
        assert np.abs(np64(gP) - rP).max() <= 1e-2 * np.abs(rP).max()
        assert np.abs(np64(gv) - rv).max() <= 1e-2 * np.abs(rv).max()

    def test_needs_input_grad_subsets(self):
        Phi, x, Y = make_inputs(2, 4, 64)
        x_t = x.detach().requires_grad_(True)
        stream_mix_add(Phi, x_t, Y).sum().backward()
        rP, rx, _, _ = omix.stream_mix_bwd(np.ones((2, 4, 64)), np64(Phi), np64(x))
        assert_rel(x_t.grad, rx, 1e-5, "grad_x only")
        P_t = Phi.detach().requires_grad_(True)
        stream_mix_add(P_t, x, Y).sum().backward()
        assert_rel(P_t.grad, rP, 1e-5, "grad_Phi only")


class TestEdgeCases:
    @pytest.mark.parametrize("D", [1, 7, 33, 100, 500])
    def test_odd_D(self, D):
        Phi, x, Y = make_inputs(1, 4, D)
        got = stream_mix_add(Phi, x, Y)
        assert_rel(got, omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y)), 1e-5, f"D={D}")

    def test_single_stream(self):
        Phi, x, Y = make_inputs(3, 1, 64)
        got = stream_mix_add(Phi, x, Y)
        assert torch.allclose(got, torch.bmm(Phi, x) + Y, atol=1e-5)

    def test_empty_batch(self):
        Phi, x, Y = make_inputs(0, 4, 64)
        assert stream_mix_add(Phi, x, Y).shape == (0, 4, 64)

    def test_cpu_raises(self):
        with pytest.raises(RuntimeError, match="CUDA"):
            stream_mix_add(torch.randn(2, 4, 4), torch.randn(2, 4, 64), torch.randn(2, 4, 64))

    def test_too_many_streams_raises(self):
        Phi, x, Y = make_inputs(2, 33, 16)
        with pytest.raises(RuntimeError, match="N <= 32"):
            stream_mix_add(Phi, x, Y)

    def test_large_D(self):
        Phi, x, Y = make_inputs(3, 8, 4096 + 8)
        got = stream_mix_add(Phi, x, Y)
        assert_rel(got, omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y)), 1e-5, "D=4104")


MIX32 = load_golden("stream_mix_f32.npz")
MIX16 = load_golden("stream_mix_f16.npz")


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in MIX32}))
def test_golden_reference_triton_fp32(case):
    """Forward and backward against outputs of the reference's own Triton
    kernels (run under the Triton interpreter on the same inputs)."""
    g = lambda name: torch.from_numpy(MIX32[f"{case}_{name}"]).to(DEVICE)  # noqa: E731
    proj = bool(MIX32[f"{case}_meta"][3])
    Phi, x, Y, Gup = g("Phi"), g("x"), g("Y"), g("Gup")
    v = g("v") if proj else None
    Phi_t, x_t, Y_t = (t.clone().requires_grad_(True) for t in (Phi, x, Y))
    v_t = v.clone().requires_grad_(True) if proj else None
    out = stream_mix_add(Phi_t, x_t, Y_t, v=v_t)
    out.backward(Gup)
    ref = lambda name: MIX32[f"{case}_{name}"].astype(np.float64)  # noqa: E731
    assert_rel(out, ref("out"), 1e-5, "out")
    assert_rel(x_t.grad, ref("gx"), 1e-5, "grad_x")
    assert_rel(Phi_t.grad, ref("gPhi"), 1e-5, "grad_Phi")
    assert torch.equal(Y_t.grad, Gup)
    if proj:
        assert_rel(v_t.grad, ref("gv"), 1e-5, "grad_v")


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in MIX16}))
def test_golden_reference_triton_fp16(case):
    g = lambda name: torch.from_numpy(MIX16[f"{case}_{name}"]).to(DEVICE)  # noqa: E731
    out = stream_mix_add(g("Phi"), g("x"), g("Y"))
    # both sides accumulate in fp32 and round once to fp16
    assert_half(out, MIX16[f"{case}_out"].astype(np.float64), "out")


@pytest.mark.parametrize("B,N,D,proj", [(3000, 4, 1024, True), (5000, 2, 2048, False), (800, 8, 4096, True),
                                        (300, 5, 2400, True), (300, 7, 1800, True), (300, 6, 1800, False),
                                        (300, 6, 512, True), (300, 8, 640, True), (300, 8, 1536, False)])
def test_many_tokens_per_cta(B, N, D, proj):
    """The pipelined kernels with many tokens per CTA, bf16 streams, repeated
    launches: forward and backward against the oracle."""
    from hyperconnections_b200 import _lib

    Phi, x, Y = make_inputs(B, N, D, dtype=torch.bfloat16)
    v = make_v(B, N) if proj else None
    torch.manual_seed(3)
    Gup = torch.randn(B, N, D).to(torch.bfloat16).to(DEVICE)
    for _ in range(3):
        P_t, x_t = Phi.detach().requires_grad_(True), x.detach().requires_grad_(True)
        v_t = v.detach().requires_grad_(True) if proj else None
        out = stream_mix_add(P_t, x_t, Y, v=v_t)
        out.backward(Gup)
    ref = omix.stream_mix_fwd(np64(Phi), np64(x), np64(Y), np64(v))
    rP, rx, _, rv = omix.stream_mix_bwd(np64(Gup), np64(Phi), np64(x), np64(v))
    assert_half(out, ref, "out")
    assert_half(x_t.grad, rx, "grad_x")
    assert np.abs(np64(P_t.grad) - rP).max() <= 1e-2 * np.abs(rP).max()
    if proj:
        assert np.abs(np64(v_t.grad) - rv).max() <= 1e-2 * np.abs(rv).max()
    assert _lib.wait_timeouts() == 0
