"""Oracle for stream mixing and the fused hyper-connection step (numpy).

Float64 accumulation of the reference's formulas; callers cast inputs from the
tensors they hold (bf16/fp16 inputs are exact in float64), so the oracle is
the exact value the reference's fp32-accumulating kernels approximate.

stream_mix_add (ops/stream_mix_small_nb.py):
  fwd  out_i = sum_j Phi_ij x_j [+ c_i (v^T x)] + Y_i,  c = v - Phi v   (:96-132)
  bwd  grad_x_j = sum_i Phi_ij G_i [+ v_j beta],  beta = c^T G          (:148-197)
       grad_Phi_ij = sum_d G_i x_eff_j,  x_eff = x - v (v^T x)          (:213-263)
       grad_v = rho - Phi^T rho + beta-part,  rho_i = sum_d G_i (v^T x),
                beta-part_n = sum_d beta x_n                            (:379-384)
fused step (cghc.py:410 read, :417 write, :449 mix), m = 1:
  fwd  u = sum_j alpha_j x_j ;  x_out_i = sum_j H_ij x_j + beta_i f
  bwd  the exact gradients of that composition.
"""

from __future__ import annotations

import numpy as np

F = np.float64


def stream_mix_fwd(Phi, x, Y, v=None):
    Phi, x, Y = (np.asarray(a, F) for a in (Phi, x, Y))
    out = np.einsum("bij,bjd->bid", Phi, x) + Y
    if v is not None:
        v = np.asarray(v, F)
        alpha = np.einsum("bn,bnd->bd", v, x)
        c = v - np.einsum("bij,bj->bi", Phi, v)
        out = out + c[:, :, None] * alpha[:, None, :]
    return out


def stream_mix_bwd(G, Phi, x, v=None):
    """Returns (grad_Phi, grad_x, grad_Y, grad_v) for upstream gradient G."""
    G, Phi, x = (np.asarray(a, F) for a in (G, Phi, x))
    grad_x = np.einsum("bij,bid->bjd", Phi, G)
    grad_v = None
    if v is None:
        grad_Phi = np.einsum("bid,bjd->bij", G, x)
    else:
        v = np.asarray(v, F)
        alpha = np.einsum("bn,bnd->bd", v, x)
        c = v - np.einsum("bij,bj->bi", Phi, v)
        beta = np.einsum("bnd,bn->bd", G, c)
        grad_x = grad_x + v[:, :, None] * beta[:, None, :]
        x_eff = x - v[:, :, None] * alpha[:, None, :]
        grad_Phi = np.einsum("bid,bjd->bij", G, x_eff)
        rho = np.einsum("bnd,bd->bn", G, alpha)
        rho_part = rho - np.einsum("bij,bi->bj", Phi, rho)
        beta_part = np.einsum("bd,bnd->bn", beta, x)
        grad_v = rho_part + beta_part
    return grad_Phi, grad_x, G, grad_v


def fused_fwd(x, f, H, alpha, beta):
    x, f, H, alpha, beta = (np.asarray(a, F) for a in (x, f, H, alpha, beta))
    u = np.einsum("tj,tjd->td", alpha, x)
    x_out = np.einsum("tij,tjd->tid", H, x) + beta[:, :, None] * f[:, None, :]
    return u, x_out


def fused_bwd(g_u, g_x, x, f, H, alpha, beta):
    """Returns (grad_x, grad_f, grad_H, grad_alpha, grad_beta)."""
    g_u, g_x, x, f, H, alpha, beta = (np.asarray(a, F) for a in (g_u, g_x, x, f, H, alpha, beta))
    grad_x = np.einsum("tij,tid->tjd", H, g_x) + alpha[:, :, None] * g_u[:, None, :]
    grad_f = np.einsum("ti,tid->td", beta, g_x)
    grad_H = np.einsum("tid,tjd->tij", g_x, x)
    grad_alpha = np.einsum("td,tjd->tj", g_u, x)
    grad_beta = np.einsum("tid,td->ti", g_x, f)
    return grad_x, grad_f, grad_H, grad_alpha, grad_beta
