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
Their autograd Functions are C++ (csrc/torch_ops.cpp, the extension
_hcops_torch.so over the C ABI): these ops are a few tens of microseconds on
the GPU, and a Python Function with ctypes launches would spend several times
that on the host.
"""

from __future__ import annotations

import torch

from .. import _lib

MAX_ORDER = 8


def _check(A: torch.Tensor, name: str) -> None:
    if A.dim() < 2 or A.shape[-1] != A.shape[-2]:
        raise ValueError(f"{name} expects (..., n, n), got shape {tuple(A.shape)}")
    if not A.is_cuda:
        raise RuntimeError(f"{name} requires CUDA tensors")
    n = A.shape[-1]
    if not 1 <= n <= MAX_ORDER:
        raise RuntimeError(f"{name} supports 1 <= n <= {MAX_ORDER}, got n={n}")


def expm_t18(A: torch.Tensor, per_matrix_scaling: bool = False) -> torch.Tensor:
    """Compute the matrix exponential of A using the T_18 Taylor approximation.

    Args:
        A: (..., n, n) float32 tensor on a CUDA device, 1 <= n <= 8.
        per_matrix_scaling: scale every matrix by its own norm instead of the
            batch maximum (the reference's behaviour, the default).

    Returns:
        exp(A) with the same shape and dtype as A.
    """
    _check(A, "expm_t18")
    return _lib.torch_ext().expm_t18(A, bool(per_matrix_scaling))


def matrix_exp(A: torch.Tensor) -> torch.Tensor:
    """exp(A) for (..., n, n), 1 <= n <= 8, by Pade [7/7] with per-matrix
    scaling and squaring; differentiable (Frechet-derivative backward)."""
    _check(A, "matrix_exp")
    return _lib.torch_ext().matrix_exp(A)
