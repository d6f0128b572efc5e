"""GPU parity tests of the batched matrix exponential (hc_expm_*).

Expected values: the CPU oracle (oracle.expm: the T18 and Pade [7/7] schemes
in float64, gradients by the block-triangular identity), outputs of the
reference's own expm_t18 body and of torch.linalg.matrix_exp (golden
fixtures), and scipy's float64 expm / expm_frechet. The parity bar is 1e-5
relative Frobenius error per matrix in fp32.
"""

import numpy as np
import pytest
import torch

from oracle import expm as oexpm
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

DEVICE = "cuda"
TOL = 1e-5


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def ops():
    from hyperconnections_b200 import ops as o

    return o


def fwd_bwd(fn, A, G):
    At = A.detach().clone().requires_grad_(True)
    E = fn(At)
    E.backward(G)
    return E.detach().cpu().numpy(), At.grad.cpu().numpy()


def config_inputs(B, n, seed=0):
    """The batched-expm workload: A = 0.5 (G - G^T) / 2 with G ~ N(0,1), then
    an upstream gradient ~ N(0,1), drawn in that order from seed 0."""
    g = torch.Generator().manual_seed(seed)
    M = torch.randn(B, n, n, generator=g)
    A = 0.5 * (M - M.mT) / 2
    G = torch.randn(B, n, n, generator=g)
    return A.to(DEVICE), G.to(DEVICE)


EXPM = load_golden("expm.npz")
KEYS = sorted({k.rsplit("_", 1)[0] for k in EXPM if k.endswith("_A")})


@pytest.mark.parametrize("key", KEYS)
def test_t18_global_matches_reference(key):
    A = torch.from_numpy(EXPM[f"{key}_A"]).to(DEVICE)
    G = torch.from_numpy(EXPM[f"{key}_G"]).to(DEVICE)
    E, dA = fwd_bwd(ops().expm_t18, A, G)
    An, Gn = EXPM[f"{key}_A"], EXPM[f"{key}_G"]
    assert oexpm.rel_fro(E, oexpm.expm_t18(An)) < TOL
    assert oexpm.rel_fro(dA, oexpm.expm_t18_grad(An, Gn)) < TOL
    # and against the reference's own float32 outputs
    assert oexpm.rel_fro(E, EXPM[f"{key}_E"]) < TOL
    assert oexpm.rel_fro(dA, EXPM[f"{key}_dA"]) < TOL


@pytest.mark.parametrize("key", KEYS)
def test_t18_per_matrix(key):
    A = torch.from_numpy(EXPM[f"{key}_A"]).to(DEVICE)
    G = torch.from_numpy(EXPM[f"{key}_G"]).to(DEVICE)
    E, dA = fwd_bwd(lambda a: ops().expm_t18(a, per_matrix_scaling=True), A, G)
    An, Gn = EXPM[f"{key}_A"], EXPM[f"{key}_G"]
    assert oexpm.rel_fro(E, oexpm.expm_t18(An, per_matrix=True)) < TOL
    assert oexpm.rel_fro(dA, oexpm.expm_t18_grad(An, Gn, per_matrix=True)) < TOL


@pytest.mark.parametrize("key", KEYS)
def test_pade_matches_torch_matrix_exp(key):
    A = torch.from_numpy(EXPM[f"{key}_A"]).to(DEVICE)
    G = torch.from_numpy(EXPM[f"{key}_G"]).to(DEVICE)
    E, dA = fwd_bwd(ops().matrix_exp, A, G)
    An, Gn = EXPM[f"{key}_A"], EXPM[f"{key}_G"]
    assert oexpm.rel_fro(E, oexpm.expm_pade(An)) < TOL
    assert oexpm.rel_fro(dA, oexpm.expm_pade_grad(An, Gn)) < TOL
    assert oexpm.rel_fro(E, EXPM[f"{key}_Em"]) < TOL
    assert oexpm.rel_fro(dA, EXPM[f"{key}_dAm"]) < TOL


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 6, 7, 8])
def test_against_exact_exponential(n):
    """Random matrices with norms spanning several scaling exponents (ragged
    batch size) against scipy's float64 expm and expm_frechet. For n = 1 the
    largest entries reach e^7: fp32 rounding of the squarings of such scalars
    alone is ~1e-5, so that case is held to 3e-5."""
    sl = pytest.importorskip("scipy.linalg")
    B = 333
    g = torch.Generator().manual_seed(n)
    A = torch.randn(B, n, n, generator=g) * torch.logspace(-3, 0.8, B).view(B, 1, 1) / n**0.5
    G = torch.randn(B, n, n, generator=g)
    An, Gn = A.double().numpy(), G.double().numpy()
    exact = np.stack([sl.expm(a) for a in An])
    dexact = np.stack([sl.expm_frechet(a.T, gg, compute_expm=False) for a, gg in zip(An, Gn)])
    tol = 3e-5 if n == 1 else TOL
    for fn in (lambda a: ops().expm_t18(a, per_matrix_scaling=True), ops().matrix_exp):
        E, dA = fwd_bwd(fn, A.to(DEVICE), G.to(DEVICE))
        assert oexpm.rel_fro(E, exact) < tol
        assert oexpm.rel_fro(dA, dexact) < tol


def test_config_batch_full_size():
    """The batched-expm workload (65,536 skew 4x4): exp of a skew matrix is
    orthogonal; every matrix against the oracle, forward and gradient."""
    A, G = config_inputs(65536, 4)
    for fn, ofwd, ograd in ((ops().expm_t18, oexpm.expm_t18, oexpm.expm_t18_grad),
                            (ops().matrix_exp, oexpm.expm_pade, oexpm.expm_pade_grad)):
        E, dA = fwd_bwd(fn, A, G)
        An, Gn = A.cpu().numpy(), G.cpu().numpy()
        assert oexpm.rel_fro(E, ofwd(An)) < TOL
        assert oexpm.rel_fro(dA, ograd(An, Gn)) < TOL
        EEt = np.einsum("bij,bkj->bik", E.astype(np.float64), E.astype(np.float64))
        assert np.abs(EEt - np.eye(4)).max() < 1e-5


def test_zero_and_identity_and_shapes():
    o = ops()
    Z = torch.zeros(5, 3, 4, 4, device=DEVICE)
    assert torch.equal(o.expm_t18(Z), torch.eye(4, device=DEVICE).expand(5, 3, 4, 4))
    assert torch.equal(o.matrix_exp(Z), torch.eye(4, device=DEVICE).expand(5, 3, 4, 4))
    assert o.expm_t18(torch.zeros(0, 4, 4, device=DEVICE)).shape == (0, 4, 4)
    # single matrix, no batch dims
    A = torch.tensor([[0.0, 1.0], [-1.0, 0.0]], device=DEVICE)
    c, s = np.cos(1.0), np.sin(1.0)
    assert np.abs(o.expm_t18(A).cpu().numpy() - np.array([[c, s], [-s, c]])).max() < 1e-6


def test_large_norm_needs_more_than_eight_squarings():
    """||A||_1 = 3000 > 3.01 * 2^8: the reference stops after 8 squarings
    (expm.py:103-104); these kernels square s = 10 times."""
    sl = pytest.importorskip("scipy.linalg")
    A = torch.tensor([[[0.0, 1500.0], [-1500.0, 0.0]]])  # rotation by 1500 rad
    exact = sl.expm(A[0].double().numpy())
    for fn in (ops().expm_t18, ops().matrix_exp):
        E = fn(A.to(DEVICE)).cpu().numpy()[0]
        # fp32 conditioning of a 1500-rad rotation limits accuracy to ~1e-4
        assert np.abs(E - exact).max() < 5e-4


def test_errors():
    o = ops()
    with pytest.raises(RuntimeError, match="CUDA"):
        o.expm_t18(torch.zeros(2, 4, 4))
    with pytest.raises(RuntimeError, match="n <= 8"):
        o.expm_t18(torch.zeros(2, 9, 9, device=DEVICE))
    with pytest.raises(ValueError):
        o.matrix_exp(torch.zeros(2, 3, 4, device=DEVICE))


def test_t18_backward_reuses_forward_partial_maxima():
    """hc_expm_t18_bwd mode 2 (the forward's partial maxima of A left in
    scratch) gives exactly the result of mode 0 (recomputed)."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(5)
    for batch, n in ((65536, 4), (3000, 7), (1, 2)):
        A = (2.0 * torch.randn(batch, n, n, generator=g)).cuda()
        G = torch.randn(batch, n, n, generator=g).cuda()
        words = lib.hc_expm_t18_scratch_words(batch, n)
        scratch = torch.empty(words, device="cuda")
        E, d0, d2 = torch.empty_like(A), torch.empty_like(A), torch.empty_like(A)
        s = torch.cuda.current_stream().cuda_stream
        _lib.check(lib.hc_expm_t18_bwd(A.data_ptr(), G.data_ptr(), d0.data_ptr(), batch, n, scratch.data_ptr(),
                                       words, 0, s), "bwd mode 0")
        scratch.fill_(float("nan"))  # mode 2 must read what the forward writes
        _lib.check(lib.hc_expm_t18_fwd(A.data_ptr(), E.data_ptr(), batch, n, scratch.data_ptr(), words, 0, s), "fwd")
        _lib.check(lib.hc_expm_t18_bwd(A.data_ptr(), G.data_ptr(), d2.data_ptr(), batch, n, scratch.data_ptr(),
                                       words, 2, s), "bwd mode 2")
        torch.cuda.synchronize()
        assert torch.equal(d0, d2)


@pytest.mark.parametrize("n", [1, 2, 3, 4])
def test_t18_forward_one_thread_per_matrix_is_bitwise_the_row_per_lane_kernel(n):
    """For n <= 4 the T18 forward runs one matrix per thread (a cooperative
    single launch when the batch fits the resident threads, else a norm pass
    and a grid-stride kernel). hc_expm_t18_fwd_noalloc still runs the
    row-per-lane kernels; the two must agree bit for bit: batch exponent 0, a
    few squarings, more than kSpecMaxS = 10 squarings (the powers formed after
    the barrier) and a batch larger than the resident threads."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(n)
    cases = [(4000, 0.2), (50000, 3.0), (3000, 2.0e4), (200000, 1.5)]
    for batch, scale in cases:
        A = (scale * torch.randn(batch, n, n, generator=g)).to(DEVICE)
        words = lib.hc_expm_t18_scratch_words(batch, n)
        scratch = torch.empty(words, device=DEVICE)
        s = torch.cuda.current_stream().cuda_stream
        E_tm, E_row = torch.empty_like(A), torch.empty_like(A)
        _lib.check(lib.hc_expm_t18_fwd(A.data_ptr(), E_tm.data_ptr(), batch, n, scratch.data_ptr(), words, 0, s),
                   "hc_expm_t18_fwd")
        _lib.check(lib.hc_expm_t18_fwd_noalloc(A.data_ptr(), E_row.data_ptr(), batch, n, s),
                   "hc_expm_t18_fwd_noalloc")
        torch.cuda.synchronize()
        finite = torch.isfinite(E_row)
        assert torch.equal(torch.isfinite(E_tm), finite)
        assert torch.equal(E_tm[finite], E_row[finite]), (batch, scale)
    assert _lib.wait_timeouts(reset=True) == 0


@pytest.mark.parametrize("n", [2, 4])
def test_t18_unaligned_buffers_take_the_scalar_path_bitwise(n):
    """Matrices of 16 and 64 bytes are read and written with 16-byte vector
    accesses when the buffers allow it; buffers that start 4 bytes off a
    16-byte boundary go through scalar accesses. Both must give the same bits
    (forward, and backward in both scaling modes)."""
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(40 + n)
    B = 5000
    A = (1.5 * torch.randn(B, n, n, generator=g)).to(DEVICE)
    G = torch.randn(B, n, n, generator=g).to(DEVICE)
    s = torch.cuda.current_stream().cuda_stream
    words = lib.hc_expm_t18_scratch_words(B, n)
    scratch = torch.empty(words, device=DEVICE)

    def off(t):  # same values, base pointer 4 bytes past a 16-byte boundary
        buf = torch.empty(t.numel() + 1, device=DEVICE)
        v = buf[1:].view(t.shape)
        v.copy_(t)
        return v

    def run(A_, G_):
        E, dA0, dA2 = (off(torch.zeros_like(A)) if A_.data_ptr() % 16 else torch.empty_like(A) for _ in range(3))
        _lib.check(lib.hc_expm_t18_fwd(A_.data_ptr(), E.data_ptr(), B, n, scratch.data_ptr(), words, 0, s), "fwd")
        _lib.check(lib.hc_expm_t18_bwd(A_.data_ptr(), G_.data_ptr(), dA2.data_ptr(), B, n, scratch.data_ptr(),
                                       words, 2, s), "bwd mode 2")
        _lib.check(lib.hc_expm_t18_bwd(A_.data_ptr(), G_.data_ptr(), dA0.data_ptr(), B, n, scratch.data_ptr(),
                                       words, 1, s), "bwd per matrix")
        torch.cuda.synchronize()
        return [t.clone() for t in (E, dA2, dA0)]

    Ao, Go = off(A), off(G)
    assert Ao.data_ptr() % 16 == 4 and A.data_ptr() % 16 == 0
    for got, want in zip(run(Ao, Go), run(A, G)):
        assert torch.equal(got, want)
    assert _lib.wait_timeouts(reset=True) == 0


@pytest.mark.parametrize("n", [2, 4, 6])
@pytest.mark.parametrize("B", [1000, 65536])
def test_global_scaling_nan_matrix_poisons_only_itself(n, B):
    """Deliberate difference from the reference: there one NaN matrix makes
    the batch maximum of ||A||_1 NaN (ops/expm.py:81-85), hence the scaling
    exponent and every output of the batch. Here the batch maximum skips NaN
    norms: the NaN matrix's own output (and gradient) is NaN, every other
    matrix gets exactly the result it gets when that matrix is zero instead
    (a zero norm never raises the maximum)."""
    A, G = config_inputs(B, n, seed=11)
    k = B // 3
    A_nan, A_zero = A.clone(), A.clone()
    A_nan[k] = float("nan")
    A_zero[k] = 0.0
    E_nan, dA_nan = fwd_bwd(ops().expm_t18, A_nan, G)
    E_zero, dA_zero = fwd_bwd(ops().expm_t18, A_zero, G)
    assert np.isnan(E_nan[k]).all() and np.isnan(dA_nan[k]).all()
    others = np.ones(B, dtype=bool)
    others[k] = False
    assert np.array_equal(E_nan[others], E_zero[others])
    assert np.array_equal(dA_nan[others], dA_zero[others])
