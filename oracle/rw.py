"""Oracle for the m-block width-read and mix + depth-write (numpy, float64).

Test infrastructure only: the parity checker of hc_read / hc_mix_write.
Float64 accumulation of the reference's formulas on the tensors' own values.

read (hyperconnections/cghc.py:410, einsum "b m n, b n d -> b m d"):
  fwd  u_k = sum_j R_kj x_j
  bwd  grad_x_j = sum_k R_kj g_k ;  grad_R_kj = sum_d g_k x_j
mix + write (cghc.py:417 einsum "b n m, b m d -> b n d", then :449
stream_mix_add, ops/stream_mix_small_nb.py:96-132 and :341-391):
  fwd  x'_i = sum_j H_ij x_j [+ c_i (v^T x)] + sum_k W_ik f_k,  c = v - H v
  bwd  the stream_mix gradients with Y = W f, plus grad_W = G f^T and
       grad_f = W^T G (the write einsum's backward).
"""

from __future__ import annotations

import numpy as np

from .stream_mix import stream_mix_bwd, stream_mix_fwd

F = np.float64


def read_fwd(R, x):
    return np.einsum("tkj,tjd->tkd", np.asarray(R, F), np.asarray(x, F))


def read_bwd(g, R, x):
    """Returns (grad_R, grad_x) for the upstream gradient g [T,m,D]."""
    g, R, x = (np.asarray(a, F) for a in (g, R, x))
    return np.einsum("tkd,tjd->tkj", g, x), np.einsum("tkj,tkd->tjd", R, g)


def mix_write_fwd(H, x, W, f, v=None):
    Y = np.einsum("tik,tkd->tid", np.asarray(W, F), np.asarray(f, F))
    return stream_mix_fwd(H, x, Y, v)


def mix_write_bwd(g, H, x, W, f, v=None):
    """Returns (grad_H, grad_x, grad_W, grad_f, grad_v) for g [T,n,D]."""
    g, W, f = (np.asarray(a, F) for a in (g, W, f))
    grad_H, grad_x, grad_Y, grad_v = stream_mix_bwd(g, H, x, v)
    grad_W = np.einsum("tid,tkd->tik", grad_Y, f)
    grad_f = np.einsum("tik,tid->tkd", W, grad_Y)
    return grad_H, grad_x, grad_W, grad_f, grad_v
