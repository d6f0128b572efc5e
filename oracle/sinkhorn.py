"""Oracle for the batched Sinkhorn-Knopp projection (numpy, float64).

Test infrastructure only: the parity checker of hc_sinkhorn_fwd/bwd.
Restates hyperconnections/mhc.py:97-102: X = exp(H), then `iters` times a row
normalisation followed by a column normalisation; the backward is reverse
mode through every step, with the iterates kept from the forward.
"""

from __future__ import annotations

import numpy as np

F = np.float64


def sinkhorn_fwd(H, iters):
    x = np.exp(np.asarray(H, F))
    for _ in range(iters):
        x = x / x.sum(-1, keepdims=True)
        x = x / x.sum(-2, keepdims=True)
    return x


def sinkhorn_bwd(H, G, iters):
    """Gradient of sum(G * sinkhorn(H)) with respect to H."""
    x0 = np.exp(np.asarray(H, F))
    ys, xs, x = [], [], x0
    for _ in range(iters):
        r = x.sum(-1, keepdims=True)
        y = x / r
        c = y.sum(-2, keepdims=True)
        x = y / c
        ys.append((y, r))
        xs.append((x, c))
    g = np.asarray(G, F)
    for k in reversed(range(iters)):
        x, c = xs[k]
        y, r = ys[k]
        g = (g - (g * x).sum(-2, keepdims=True)) / c
        g = (g - (g * y).sum(-1, keepdims=True)) / r
    return g * x0
