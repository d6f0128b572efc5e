"""Batched small-matrix exponential, drop-in for ``hyperconnections.ops.expm``.

``expm_t18(A)`` keeps the reference's algorithm and signature
(hyperconnections/ops/expm.py:65-106): the optimised degree-18 Taylor
polynomial of Bader, Blanes and Casas (2019) with scaling and squaring and ONE
scaling exponent for the whole batch, from max ||A||_1 (expm.py:81-85). For
n <= 4 the forward is one cooperative kernel launch (the batch maximum, a
grid barrier and T18 in one kernel; larger batches or n take a batch-max
kernel first); the backward is one launch that reuses the forward's partial
maxima, the adjoint Frechet derivative of the same approximant (what the
reference gets from autograd through its graph).

Differences from the reference, both deliberate:
* the squaring loop runs s times; the reference stops after 8 squarings
  (expm.py:103-104), which is wrong once max ||A||_1 > 3.01 * 2^8;
* ``per_matrix_scaling=True`` gives every matrix its own exponent.

``matrix_exp(A)`` replaces ``torch.linalg.matrix_exp`` where CGHC builds its
transition matrices (cghc.py:321): diagonal Pade [7/7] with per-matrix scaling
and squaring (Higham 2005) and its Frechet-derivative backward (Al-Mohy and
Higham 2009).

Both take (..., n, n) with 1 <= n <= 8 on a CUDA device. Inputs that are not
float32 are computed in float32 and the result is cast back to their dtype.
"""

from __future__ import annotations

import torch

from .. import _lib

MAX_ORDER = 8


def _flatten(A: torch.Tensor, name: str):
    if A.dim() < 2 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"{name} expects (..., n, n), got shape {tuple(A.shape)}")
    if not A.is_cuda:
        raise RuntimeError(f"{name} requires CUDA tensors")
    n = A.shape[-1]
    if not 1 <= n <= MAX_ORDER:
        raise RuntimeError(f"{name} supports 1 <= n <= {MAX_ORDER}, got n={n}")
    if A.dtype != torch.float32:
        A = A.to(torch.float32)
    if not A.is_contiguous():
        A = A.contiguous()
    return A.view(-1, n, n), n


_SCRATCH_WORDS: dict = {}


def _scratch_words(batch: int, n: int, device_index: int) -> int:
    """Floats of global-scaling scratch for (batch, n) on a device (depends
    on the device's occupancy; cached)."""
    key = (batch, n, device_index)
    words = _SCRATCH_WORDS.get(key)
    if words is None:
        words = max(1, int(_lib.lib().hc_expm_t18_scratch_words(batch, n)))
        if len(_SCRATCH_WORDS) < 4096:
            _SCRATCH_WORDS[key] = words
    return words


def _restore(t: torch.Tensor, shape, dtype) -> torch.Tensor:
    t = t.view(shape)
    return t if dtype == torch.float32 else t.to(dtype)


class _ExpmT18Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, per_matrix):
        A32, n = _flatten(A, "expm_t18")
        batch = A32.shape[0]
        size = batch * n * n
        buf = None
        if per_matrix:
            E = torch.empty_like(A32)
            scratch_ptr, words = None, 0
        else:
            # one allocation: E, then the partial maxima the backward reuses
            words = _scratch_words(batch, n, A32.device.index)
            buf = torch.empty(size + words, dtype=torch.float32, device=A32.device)
            E = buf[:size].view(batch, n, n)
            scratch_ptr = buf.data_ptr() + 4 * size
        with _lib.on_device(A32):
            rc = _lib.lib().hc_expm_t18_fwd(A32.data_ptr(), E.data_ptr(), batch, n, scratch_ptr, words,
                                            1 if per_matrix else 0, _lib.stream_of(A32))
        _lib.check(rc, "hc_expm_t18_fwd")
        ctx.save_for_backward(A32)
        ctx.keep = buf  # holds the partial maxima the backward reuses
        ctx.scratch = (scratch_ptr, words)
        ctx.per_matrix = per_matrix
        ctx.shape = A.shape
        ctx.dtype = A.dtype
        return _restore(E, A.shape, A.dtype)

    @staticmethod
    def backward(ctx, grad):
        (A32,) = ctx.saved_tensors
        batch, n, _ = A32.shape
        G = grad if grad.dtype == torch.float32 else grad.to(torch.float32)
        G = (G if G.is_contiguous() else G.contiguous()).view(batch, n, n)
        dA = torch.empty_like(A32)
        scratch_ptr, words = ctx.scratch
        with _lib.on_device(A32):
            rc = _lib.lib().hc_expm_t18_bwd(A32.data_ptr(), G.data_ptr(), dA.data_ptr(), batch, n, scratch_ptr,
                                            words, 1 if ctx.per_matrix else 2, _lib.stream_of(A32))
        _lib.check(rc, "hc_expm_t18_bwd")
        return _restore(dA, ctx.shape, ctx.dtype), None


class _ExpmPadeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A):
        A32, n = _flatten(A, "matrix_exp")
        batch = A32.shape[0]
        E = torch.empty_like(A32)
        with _lib.on_device(A32):
            rc = _lib.lib().hc_expm_pade_fwd(A32.data_ptr(), E.data_ptr(), batch, n, _lib.stream_of(A32))
        _lib.check(rc, "hc_expm_pade_fwd")
        ctx.save_for_backward(A32)
        ctx.shape = A.shape
        ctx.dtype = A.dtype
        return _restore(E, A.shape, A.dtype)

    @staticmethod
    def backward(ctx, grad):
        (A32,) = ctx.saved_tensors
        batch, n, _ = A32.shape
        G = grad if grad.dtype == torch.float32 else grad.to(torch.float32)
        G = (G if G.is_contiguous() else G.contiguous()).view(batch, n, n)
        dA = torch.empty_like(A32)
        with _lib.on_device(A32):
            rc = _lib.lib().hc_expm_pade_bwd(A32.data_ptr(), G.data_ptr(), dA.data_ptr(), batch, n,
                                             _lib.stream_of(A32))
        _lib.check(rc, "hc_expm_pade_bwd")
        return _restore(dA, ctx.shape, ctx.dtype)


def expm_t18(A: torch.Tensor, per_matrix_scaling: bool = False) -> torch.Tensor:
    """Compute the matrix exponential of A using the T_18 Taylor approximation.

    Args:
        A: (..., n, n) float32 tensor on a CUDA device, 1 <= n <= 8.
        per_matrix_scaling: scale every matrix by its own norm instead of the
            batch maximum (the reference's behaviour, the default).

    Returns:
        exp(A) with the same shape and dtype as A.
    """
    return _ExpmT18Fn.apply(A, bool(per_matrix_scaling))


def matrix_exp(A: torch.Tensor) -> torch.Tensor:
    """exp(A) for (..., n, n), 1 <= n <= 8, by Pade [7/7] with per-matrix
    scaling and squaring; differentiable (Frechet-derivative backward)."""
    return _ExpmPadeFn.apply(A)
