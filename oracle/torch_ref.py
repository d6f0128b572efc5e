"""The reference's eager PyTorch CPU path for the hot-path work — the timed
CPU baseline (bench.py's cpu_baseline leg and ``--impl reference``).

These functions restate, op for op, what the reference runs on a CPU:

* ``fused_step_cpu``: CGHC's read einsum (cghc.py:410), write einsum
  (cghc.py:417) and eager stream mix (cghc.py:365-392, no projection: einsum
  then + Y) under bf16 autocast, as the reference trains (experiments/cifar.py:
  272), followed by the autograd backward with the given upstream gradients.
  On CPU the reference's Triton path raises (ops/stream_mix.py:76-77), so the
  eager path is the one CGHC runs there.
* ``expm_t18_cpu``: the body of expm_t18 (ops/expm.py:81-106) run eagerly
  (its torch.compile wrapper does not build on this CPU), forward + autograd
  backward.
"""

from __future__ import annotations

import torch

from .expm import (A11, A21, A31, B02, B03, B11, B12, B13, B21, B22, B23, B24, B31, B32, B33, B34,
                   B61, B62, B63, B64, THETA_18)


def fused_step_cpu(x, f, H, alpha, beta, g_u, g_x):
    """Forward + backward of the fused step on CPU tensors; returns
    (u, x_out, grad_x, grad_f, grad_H, grad_alpha, grad_beta)."""
    x = x.detach().requires_grad_(True)
    f = f.detach().requires_grad_(True)
    H = H.detach().requires_grad_(True)
    alpha = alpha.detach().requires_grad_(True)
    beta = beta.detach().requires_grad_(True)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        u = torch.einsum("bmn,bnd->bmd", alpha[:, None, :], x)            # cghc.py:410
        Y = torch.einsum("bnm,bmd->bnd", beta[:, :, None], f[:, None, :])  # cghc.py:417
        x_mixed = torch.einsum("bij,bjd->bid", H, x)                       # cghc.py:373-375
        out = x_mixed + Y                                                  # cghc.py:392
    torch.autograd.backward([u, out], [g_u[:, None, :].to(u.dtype), g_x.to(out.dtype)])
    return u[:, 0], out, x.grad, f.grad, H.grad, alpha.grad, beta.grad


def expm_t18_cpu(A: torch.Tensor, G: torch.Tensor):
    """Eager expm_t18 body with autograd; returns (E, dA)."""
    A = A.detach().requires_grad_(True)
    with torch.no_grad():
        nrm = torch.linalg.matrix_norm(A, ord=1).max().clamp_min(THETA_18)
        s = torch.ceil(torch.log2(nrm / THETA_18)).clamp(min=0)
        scale = 2.0**s
    As = A / scale
    eye = torch.eye(A.shape[-1], dtype=A.dtype)
    A2 = As @ As
    A3 = A2 @ As
    A6 = A3 @ A3
    Bm1 = A11 * As + A21 * A2 + A31 * A3
    Bm2 = B11 * As + B21 * A2 + B31 * A3 + B61 * A6
    Bm3 = B02 * eye + B12 * As + B22 * A2 + B32 * A3 + B62 * A6
    Bm4 = B03 * eye + B13 * As + B23 * A2 + B33 * A3 + B63 * A6
    Bm5 = B24 * A2 + B34 * A3 + B64 * A6
    A9 = Bm1 @ Bm5 + Bm4
    T = Bm2 + (Bm3 + A9) @ A9
    for i in range(8):
        T = torch.where(s > i, T @ T, T)
    T.backward(G)
    return T.detach(), A.grad
