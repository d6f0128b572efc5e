"""Pins the CPU oracle against outputs of the reference's own code
(tests/golden/*.npz, made by tests/golden/make_golden.py). CPU only."""

import numpy as np
import pytest

from oracle import expm as oexpm
from oracle import rw as orw
from oracle import stream_mix as omix
from tests.conftest import load_golden

EXPM = load_golden("expm.npz")
MIX32 = load_golden("stream_mix_f32.npz")
MIX16 = load_golden("stream_mix_f16.npz")
FUSED = load_golden("fused.npz")
RW = load_golden("rw.npz")

EXPM_KEYS = sorted({k.rsplit("_", 1)[0] for k in EXPM if k.endswith("_A")})


@pytest.mark.parametrize("key", EXPM_KEYS)
def test_oracle_expm_t18_matches_reference(key):
    A, G = EXPM[f"{key}_A"], EXPM[f"{key}_G"]
    E = oexpm.expm_t18(A)
    dA = oexpm.expm_t18_grad(A, G)
    # reference runs the same scheme in float32; the oracle in float64
    assert oexpm.rel_fro(E, EXPM[f"{key}_E"]) < 1e-5
    assert oexpm.rel_fro(dA, EXPM[f"{key}_dA"]) < 1e-5


@pytest.mark.parametrize("key", EXPM_KEYS)
def test_oracle_pade_matches_torch_matrix_exp(key):
    A, G = EXPM[f"{key}_A"], EXPM[f"{key}_G"]
    assert oexpm.rel_fro(oexpm.expm_pade(A), EXPM[f"{key}_Em"]) < 1e-5
    assert oexpm.rel_fro(oexpm.expm_pade_grad(A, G), EXPM[f"{key}_dAm"]) < 1e-5


@pytest.mark.parametrize("key", EXPM_KEYS)
def test_oracle_approximants_match_exact_exponential(key):
    """T18 and Pade [7/7] agree with scipy's float64 expm / expm_frechet to
    far below the 1e-5 parity tolerance."""
    scipy_linalg = pytest.importorskip("scipy.linalg")
    A, G = EXPM[f"{key}_A"].astype(np.float64), EXPM[f"{key}_G"].astype(np.float64)
    exact = np.stack([scipy_linalg.expm(a) for a in A])
    dexact = np.stack([scipy_linalg.expm_frechet(a.T, g, compute_expm=False) for a, g in zip(A, G)])
    assert oexpm.rel_fro(oexpm.expm_t18(A), exact) < 1e-6
    assert oexpm.rel_fro(oexpm.expm_pade(A), exact) < 1e-6
    assert oexpm.rel_fro(oexpm.expm_t18_grad(A, G), dexact) < 1e-6
    assert oexpm.rel_fro(oexpm.expm_pade_grad(A, G), dexact) < 1e-6


def test_scaling_exponent_matches_reference_rule():
    # s = ceil(log2(norm / 3.01)) clamped at 0 (reference expm.py:81-85)
    norms = np.array([0.0, 1.0, 3.01, 3.02, 6.02, 6.03, 770.0, 1e6], dtype=np.float32)
    want = [0, 0, 0, 1, 1, 2, 8, 19]
    assert oexpm.scaling_exponent(norms, oexpm.THETA_18).tolist() == want


MIX_CASES = sorted({k.split("_")[0] for k in MIX32})


@pytest.mark.parametrize("case", MIX_CASES)
def test_oracle_stream_mix_matches_reference_triton(case):
    g = lambda name: MIX32[f"{case}_{name}"]  # noqa: E731
    proj = bool(g("meta")[3])
    v = g("v") if proj else None
    out = omix.stream_mix_fwd(g("Phi"), g("x"), g("Y"), v)
    np.testing.assert_allclose(out, g("out"), rtol=1e-5, atol=1e-5)
    gPhi, gx, gY, gv = omix.stream_mix_bwd(g("Gup"), g("Phi"), g("x"), v)
    np.testing.assert_allclose(gx, g("gx"), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gPhi, g("gPhi"), rtol=1e-4, atol=1e-4)
    np.testing.assert_array_equal(gY, g("gY"))
    if proj:
        np.testing.assert_allclose(gv, g("gv"), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in MIX16}))
def test_oracle_stream_mix_fp16_matches_reference(case):
    g = lambda name: MIX16[f"{case}_{name}"]  # noqa: E731
    out = omix.stream_mix_fwd(g("Phi"), g("x"), g("Y"))
    np.testing.assert_allclose(out, g("out").astype(np.float64), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in FUSED}))
def test_oracle_fused_matches_reference_composition(case):
    g = lambda name: FUSED[f"{case}_{name}"]  # noqa: E731
    u, x_out = omix.fused_fwd(g("x"), g("f"), g("H"), g("alpha"), g("beta"))
    np.testing.assert_allclose(u, g("u"), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(x_out, g("x_out"), rtol=1e-5, atol=1e-5)
    grads = omix.fused_bwd(g("g_u"), g("g_x"), g("x"), g("f"), g("H"), g("alpha"), g("beta"))
    for name, got in zip(("grad_x", "grad_f", "grad_H", "grad_alpha", "grad_beta"), grads):
        np.testing.assert_allclose(got, g(name), rtol=1e-4, atol=1e-4, err_msg=name)


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in RW}))
def test_oracle_read_mix_write_matches_reference(case):
    """m-block read (einsum, cghc.py:410) and write + mix (:417, :449), with
    and without the projection direction."""
    g = lambda name: RW[f"{case}_{name}"]  # noqa: E731
    proj = bool(g("meta")[4])
    v = g("v") if proj else None
    np.testing.assert_allclose(orw.read_fwd(g("R"), g("x")), g("u"), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(orw.mix_write_fwd(g("H"), g("x"), g("W"), g("f"), v), g("x_out"),
                               rtol=1e-5, atol=1e-5)
    gR, gx_read = orw.read_bwd(g("g_u"), g("R"), g("x"))
    gH, gx_mix, gW, gf, gv = orw.mix_write_bwd(g("g_x"), g("H"), g("x"), g("W"), g("f"), v)
    np.testing.assert_allclose(gx_read + gx_mix, g("grad_x"), rtol=1e-4, atol=1e-4)
    for name, got in (("grad_R", gR), ("grad_W", gW), ("grad_f", gf), ("grad_H", gH)):
        np.testing.assert_allclose(got, g(name), rtol=1e-4, atol=1e-4, err_msg=name)
    if proj:
        np.testing.assert_allclose(gv, g("grad_v"), rtol=1e-4, atol=1e-4)


LAYER = load_golden("layer.npz")
LAYER_CASES = sorted({k.split("_")[0] for k in LAYER})


def layer_chain_oracle(g):
    """Float64 oracle of one CGHC layer's chain: read -> Linear -> write ->
    matrix_exp -> mix, forward and backward (cghc.py:321, :410, :417, :449)."""
    x, R, W, A, G = g("x"), g("read_in"), g("write_out"), g("A"), g("g")
    Wm, bm = g("W_mod").astype(np.float64), g("b_mod").astype(np.float64)
    T, n, block = x.shape
    m = R.shape[1]
    v = g("v") if bool(g("meta")[5]) else None
    vt = None if v is None else np.broadcast_to(v, (T, n))
    Phi = np.stack([oexpm.expm_pade(a[None])[0] for a in A.astype(np.float64)])
    u = orw.read_fwd(R, x)
    f = (u.reshape(T, m * block) @ Wm.T + bm).reshape(T, m, block)
    out = orw.mix_write_fwd(Phi, x, W, f, vt)
    gPhi, gx_mix, gW, gf, gv = orw.mix_write_bwd(G, Phi, x, W, f, vt)
    gf_flat = gf.reshape(T, m * block)
    grads = {
        "grad_W_mod": gf_flat.T @ u.reshape(T, m * block),
        "grad_b_mod": gf_flat.sum(0),
        "grad_write_out": gW,
        "grad_A": oexpm.expm_pade_grad(A.astype(np.float64), gPhi),
    }
    gR, gx_read = orw.read_bwd((gf_flat @ Wm).reshape(T, m, block), R, x)
    grads["grad_read_in"] = gR
    grads["grad_x"] = gx_mix + gx_read
    if v is not None:
        grads["grad_v"] = gv.sum(0, keepdims=True) if v.shape[0] == 1 else gv
    return out, grads


@pytest.mark.parametrize("case", LAYER_CASES)
def test_oracle_cghc_layer_chain_matches_reference(case):
    g = lambda name: LAYER[f"{case}_{name}"]  # noqa: E731
    out, grads = layer_chain_oracle(g)
    scale = lambda r: max(1.0, np.abs(r).max())  # noqa: E731
    assert np.abs(out - g("out")).max() <= 1e-5 * scale(g("out"))
    for name, got in grads.items():
        ref = g(name)
        assert np.abs(got - ref).max() <= 1e-5 * scale(ref), name


SINK = load_golden("sinkhorn.npz")


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in SINK}))
def test_oracle_sinkhorn_matches_reference(case):
    """MHC's Sinkhorn-Knopp method (mhc.py:97-102), forward and autograd backward."""
    from oracle import sinkhorn as osk

    g = lambda name: SINK[f"{case}_{name}"]  # noqa: E731
    iters = int(g("meta")[2])
    np.testing.assert_allclose(osk.sinkhorn_fwd(g("H"), iters), g("P"), rtol=1e-5, atol=1e-6)
    dH = osk.sinkhorn_bwd(g("H"), g("G"), iters)
    assert np.abs(dH - g("dH")).max() <= 1e-5 * max(1.0, np.abs(g("dH")).max())


MIXL = load_golden("stream_mix_large_n.npz")


@pytest.mark.parametrize("case", sorted({k.split("_")[0] for k in MIXL}))
def test_oracle_stream_mix_large_n_matches_reference(case):
    g = lambda name: MIXL[f"{case}_{name}"]  # noqa: E731
    proj = bool(g("meta")[3])
    v = g("v") if proj else None
    np.testing.assert_allclose(omix.stream_mix_fwd(g("Phi"), g("x"), g("Y"), v), g("out"), rtol=1e-5, atol=1e-5)
    gP, gx, _, gv = omix.stream_mix_bwd(g("Gup"), g("Phi"), g("x"), v)
    np.testing.assert_allclose(gP, g("gPhi"), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(gx, g("gx"), rtol=1e-4, atol=1e-4)
    if proj:
        np.testing.assert_allclose(gv, g("gv"), rtol=1e-4, atol=1e-4)


GEN = load_golden("generator.npz")
GEN_CASES = sorted({k.split("_")[0] for k in GEN})
GEN_INPUTS = ("M", "lc", "R", "dpre", "S", "ld")


def generator_oracle(case):
    """A and the gradients of sum(G * A) from oracle.generator (float64)."""
    import torch

    from oracle import generator as ogen

    g = lambda name: GEN[f"{case}_{name}"]  # noqa: E731
    vec = bool(g("meta")[1])
    ins = {k: torch.tensor(g(k), dtype=torch.float64, requires_grad=True) for k in GEN_INPUTS
           if f"{case}_{k}" in GEN}
    A = ogen.generator(**ins, ranges=tuple(g("ranges")), vec_dt=vec)
    A.backward(torch.tensor(g("G"), dtype=torch.float64))
    return A.detach().numpy(), {k: v.grad.numpy() for k, v in ins.items()}


@pytest.mark.parametrize("case", GEN_CASES)
def test_oracle_generator_matches_reference(case):
    A, grads = generator_oracle(case)
    ref = GEN[f"{case}_A"]
    assert np.abs(A - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), str(GEN[f"{case}_type"])
    for k, got in grads.items():
        want = GEN[f"{case}_d{k}"]
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), (str(GEN[f"{case}_type"]), k)
