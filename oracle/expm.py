"""Oracle for the batched matrix exponential (numpy, float64 by default).

Restates hyperconnections/ops/expm.py:65-106 (expm_t18) — the optimised
degree-18 Taylor polynomial of Bader, Blanes and Casas, Mathematics 7 (2019)
1174, eq. (15), with scaling and squaring at theta_18 = 3.01 — and the diagonal
Pade [7/7] approximant of Higham (2005) used by the B200 ``matrix_exp``.

Gradients use the block-triangular identity: for a polynomial or rational f
with real coefficients, f([[X, E], [0, X]]) = [[f(X), L_f(X, E)], [0, f(X)]],
and the gradient of sum(G * f(A)) is L_f(A^T, G). The scaling exponent is held
fixed at the forward's value, so the result is the derivative of the same
approximant the reference differentiates with autograd.
"""

from __future__ import annotations

import numpy as np

# Bader, Blanes, Casas (2019) eq. (15) coefficients (reference expm.py:27-59).
A01, A11, A21, A31 = 0.0, -0.10036558103014462, -0.008029246482411570, -0.000892138498045730
B01, B11, B21, B31, B61 = 0.0, 0.39784974949645076, 1.36783778460411719, 0.49828962252538268, -0.00063789819459247233
B02, B12, B22, B32, B62 = -10.96763960529620626, 1.68015813878906197, 0.05717798464788655, -0.00698210122488052, 0.00003349750170860705
B03, B13, B23, B33, B63 = -0.09043168323908106, -0.06764045190713819, 0.06759613017740597, 0.02955525704293155, -0.00001391802575160607
B04, B14, B24, B34, B64 = 0.0, 0.0, -0.09233646193671186, -0.01693649390020817, -0.00001400867981820361
THETA_18 = 3.01
# Higham (2005), single precision: theta_7 for the [7/7] Pade approximant.
THETA_7 = 3.925724783138660
PADE7 = (17297280.0, 8648640.0, 1995840.0, 277200.0, 25200.0, 1512.0, 56.0, 1.0)


def norm1(A: np.ndarray) -> np.ndarray:
    """Per-matrix 1-norm (max column sum), computed in float32 like the GPU."""
    return np.abs(A.astype(np.float32)).sum(axis=-2, dtype=np.float32).max(axis=-1)


def scaling_exponent(norm, theta: float) -> np.ndarray:
    """ceil(log2(norm/theta)) clamped at 0 (reference expm.py:81-85), from the
    float32 quotient, evaluated exactly."""
    norm = np.asarray(norm, dtype=np.float32)
    ratio = (norm / np.float32(theta)).astype(np.float32)
    out = np.zeros(ratio.shape, dtype=np.int64)
    big = norm > np.float32(theta)
    m, e = np.frexp(ratio[big].astype(np.float64))  # ratio = m * 2^e, m in [0.5, 1)
    out[big] = np.where(m == 0.5, e - 1, e)
    return out


def _eye_like(A):
    n = A.shape[-1]
    return np.broadcast_to(np.eye(n, dtype=A.dtype), A.shape)


def t18_poly(A: np.ndarray) -> np.ndarray:
    """The T18 evaluation scheme (reference expm.py:88-99), batched."""
    I = _eye_like(A)
    A2 = A @ A
    A3 = A2 @ A
    A6 = A3 @ A3
    Bm1 = A01 * I + A11 * A + A21 * A2 + A31 * A3
    Bm2 = B01 * I + B11 * A + B21 * A2 + B31 * A3 + B61 * A6
    Bm3 = B02 * I + B12 * A + B22 * A2 + B32 * A3 + B62 * A6
    Bm4 = B03 * I + B13 * A + B23 * A2 + B33 * A3 + B63 * A6
    Bm5 = B04 * I + B14 * A + B24 * A2 + B34 * A3 + B64 * A6
    A9 = Bm1 @ Bm5 + Bm4
    return Bm2 + (Bm3 + A9) @ A9


def pade7_rat(A: np.ndarray) -> np.ndarray:
    """r_7(A) = q(A)^{-1} p(A) for the [7/7] Pade approximant."""
    b = PADE7
    I = _eye_like(A)
    A2 = A @ A
    A4 = A2 @ A2
    A6 = A4 @ A2
    U = A @ (b[7] * A6 + b[5] * A4 + b[3] * A2 + b[1] * I)
    V = b[6] * A6 + b[4] * A4 + b[2] * A2 + b[0] * I
    return np.linalg.solve(V - U, V + U)


def _apply(f, A: np.ndarray, s: np.ndarray) -> np.ndarray:
    """f(A / 2^s)^(2^s) with a per-matrix exponent array s (broadcast)."""
    s = np.broadcast_to(np.asarray(s), A.shape[:-2])
    scale = np.ldexp(1.0, -s).astype(A.dtype)[..., None, None]
    X = f(A * scale)
    for i in range(int(s.max()) if s.size else 0):
        X = np.where((s > i)[..., None, None], X @ X, X)
    return X


def t18_exponents(A: np.ndarray, per_matrix: bool) -> np.ndarray:
    nrm = norm1(A)
    if per_matrix:
        return scaling_exponent(nrm, THETA_18)
    return np.full(A.shape[:-2], scaling_exponent(nrm.max() if nrm.size else 0.0, THETA_18), dtype=np.int64)


def expm_t18(A: np.ndarray, per_matrix: bool = False, dtype=np.float64) -> np.ndarray:
    """exp(A) by the reference's T18 scheme (global exponent by default)."""
    s = t18_exponents(A, per_matrix)
    return _apply(t18_poly, A.astype(dtype), s)


def _block(At: np.ndarray, G: np.ndarray) -> np.ndarray:
    n = At.shape[-1]
    M = np.zeros(At.shape[:-2] + (2 * n, 2 * n), dtype=At.dtype)
    M[..., :n, :n] = At
    M[..., n:, n:] = At
    M[..., :n, n:] = G
    return M


def expm_t18_grad(A: np.ndarray, G: np.ndarray, per_matrix: bool = False, dtype=np.float64) -> np.ndarray:
    """Gradient of sum(G * expm_t18(A)) w.r.t. A = L(A^T, G) of the approximant."""
    n = A.shape[-1]
    s = t18_exponents(A, per_matrix)
    M = _block(np.swapaxes(A, -1, -2).astype(dtype), G.astype(dtype))
    return _apply(t18_poly, M, s)[..., :n, n:]


def pade_exponents(A: np.ndarray) -> np.ndarray:
    return scaling_exponent(norm1(A), THETA_7)


def expm_pade(A: np.ndarray, dtype=np.float64) -> np.ndarray:
    return _apply(pade7_rat, A.astype(dtype), pade_exponents(A))


def expm_pade_grad(A: np.ndarray, G: np.ndarray, dtype=np.float64) -> np.ndarray:
    n = A.shape[-1]
    M = _block(np.swapaxes(A, -1, -2).astype(dtype), G.astype(dtype))
    return _apply(pade7_rat, M, pade_exponents(A))[..., :n, n:]


def rel_fro(got: np.ndarray, ref: np.ndarray) -> float:
    """max over matrices of ||got - ref||_F / max(||ref||_F, tiny)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    num = np.sqrt(((got - ref) ** 2).sum(axis=(-2, -1)))
    den = np.maximum(np.sqrt((ref**2).sum(axis=(-2, -1))), 1e-30)
    return float((num / den).max()) if num.size else 0.0
