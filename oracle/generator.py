"""Oracle for CGHC's generator assembly (torch on the CPU, float64).

Test infrastructure only: the parity checker of hc_cghc_generator_fwd/bwd.
Restates hyperconnections/cghc.py:219-315 from the pre-activations (the
module's Linear outputs plus its static parameters) step by step; the
gradient is autograd through this restatement.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _sandwich(X, dt, vec_dt):
    """dt * X for a scalar dt, sqrt(dt_i) X_ij sqrt(dt_j) per stream (cghc.py:245-251)."""
    if not vec_dt:
        return dt.unsqueeze(-1) * X
    s = dt.sqrt()
    return s[..., :, None] * X * s[..., None, :]


def generator(M=None, lc=None, R=None, dpre=None, S=None, ld=None, ranges=(0.001, 1.0, 0.001, 1.0),
              vec_dt=False):
    lo_c, hi_c, lo_d, hi_d = ranges
    ref = next(t for t in (M, R, S) if t is not None) if any(t is not None for t in (M, R, S)) else None
    n = ref.shape[-1] if ref is not None else dpre.shape[-1]
    lead = (ref.shape[:-2] if ref is not None else dpre.shape[:-1])
    A = torch.zeros(*lead, n, n, dtype=torch.float64)
    if M is not None:
        dt = lo_c + (hi_c - lo_c) * torch.sigmoid(lc)
        A = A + _sandwich(M - M.transpose(-1, -2), dt, vec_dt)
    if ld is not None:
        dt_d = lo_d + (hi_d - lo_d) * torch.sigmoid(ld)
        if R is not None:
            A = A - _sandwich(R @ R.transpose(-1, -2) / math.sqrt(n), dt_d, vec_dt)
        if dpre is not None:
            A = A - torch.diag_embed(dt_d * F.softplus(dpre))
        if S is not None:
            sym = 0.5 * (S + S.transpose(-1, -2))
            adj = F.softplus(sym)
            adj = adj - torch.diag_embed(torch.diagonal(adj, dim1=-2, dim2=-1))
            lap = torch.diag_embed(adj.sum(-1)) - adj
            A = A - _sandwich(lap, dt_d, vec_dt)
    return A
