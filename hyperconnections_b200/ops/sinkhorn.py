"""Batched Sinkhorn-Knopp projection, drop-in for MHC's ``_sinkhorn_knopp``
(hyperconnections/mhc.py:97-102): exp of the logits, then ``iters`` rounds of
row normalisation followed by column normalisation, per n x n matrix.

One kernel launch for the forward and one for the backward, each matrix in
one thread's registers; the reference runs 1 + 4 * iters elementwise and
reduction ops per direction and keeps every intermediate for autograd.

``sinkhorn_knopp(logits, iters=20)``: logits (..., n, n) with n <= 8 on a
CUDA device, computed in float32 and returned in the logits' dtype.
"""

from __future__ import annotations

import torch

from .. import _lib

MAX_ORDER = 8
MAX_ITERS = 256


class _SinkhornFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, H, iters):
        n = H.shape[-1]
        H32 = H.to(torch.float32).contiguous().view(-1, n, n)
        P = torch.empty_like(H32)
        batch = H32.shape[0]
        with _lib.on_device(H):
            rc = _lib.lib().hc_sinkhorn_fwd(H32.data_ptr(), P.data_ptr(), batch, n, iters, _lib.stream_of(H32))
        _lib.check(rc, "hc_sinkhorn_fwd")
        ctx.save_for_backward(H32)
        ctx.iters, ctx.shape, ctx.dtype = iters, H.shape, H.dtype
        return P.view(H.shape).to(H.dtype)

    @staticmethod
    def backward(ctx, grad):
        (H32,) = ctx.saved_tensors
        batch, n, _ = H32.shape
        G = grad.to(torch.float32).contiguous().view(batch, n, n)
        dH = torch.empty_like(H32)
        with _lib.on_device(H32):
            rc = _lib.lib().hc_sinkhorn_bwd(H32.data_ptr(), G.data_ptr(), dH.data_ptr(), batch, n, ctx.iters,
                                            _lib.stream_of(H32))
        _lib.check(rc, "hc_sinkhorn_bwd")
        return dH.view(ctx.shape).to(ctx.dtype), None


def sinkhorn_knopp(logits: torch.Tensor, iters: int = 20) -> torch.Tensor:
    """Doubly stochastic projection of exp(logits) (see module doc)."""
    if not _lib.available():
        raise RuntimeError("sinkhorn_knopp requires the hyperconnections_b200 CUDA kernels (libhcops.so)")
    if not logits.is_cuda:
        raise RuntimeError("sinkhorn_knopp requires CUDA tensors")
    if logits.dim() < 2 or logits.shape[-1] != logits.shape[-2]:
        raise ValueError(f"sinkhorn_knopp expects (..., n, n), got shape {tuple(logits.shape)}")
    n = logits.shape[-1]
    if not 1 <= n <= MAX_ORDER:
        raise RuntimeError(f"sinkhorn_knopp supports 1 <= n <= {MAX_ORDER}, got n={n}")
    if not 0 <= iters <= MAX_ITERS:
        raise RuntimeError(f"sinkhorn_knopp supports 0 <= iters <= {MAX_ITERS}, got {iters}")
    return _SinkhornFn.apply(logits, int(iters))
