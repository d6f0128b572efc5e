"""Half-precision parity bound shared by the GPU tests.

A bf16 / fp16 output of the stream-mixing kernels is an fp32-accumulated sum
rounded once to the stream dtype. It is compared elementwise with a float64
oracle (or an fp32 reference fixture) computed from the same half-precision
inputs:

* where |ref| < 8:   |got - ref| <= 2e-2 (bf16) or 1e-2 (fp16), the absolute
  bar of the parity target. A correctly rounded result stays within half an
  ulp there (at most 2^-6 = 0.0156 in bf16, 2^-9 in fp16), so this leaves no
  room for a second rounding or a half-precision accumulation;
* where |ref| >= 8:  |got - ref| <= half-ulp(ref) + the same absolute bar,
  because the output rounding alone can exceed 2e-2 there (bf16 half-ulp is
  2^-5 at 8 <= |ref| < 16). These elements are counted and reported
  separately instead of being folded into a looser bound for every element.
"""

from __future__ import annotations

import numpy as np
import torch

HALF_ATOL = {torch.bfloat16: 2e-2, torch.float16: 1e-2}
_MANTISSA_BITS = {torch.bfloat16: 7, torch.float16: 10}
LARGE = 8.0


def half_ulp(ref: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Half the spacing of `dtype` values at |ref| (normal range)."""
    _, k = np.frexp(np.abs(ref))  # |ref| = m 2^k, 0.5 <= m < 1: the binade is [2^(k-1), 2^k)
    return np.ldexp(1.0, k - 1 - _MANTISSA_BITS[dtype] - 1)


def assert_half(got, ref: np.ndarray, what: str = "", dtype: torch.dtype | None = None) -> int:
    """Assert the bound above for a half-precision result; returns how many
    elements had |ref| >= 8 (reported in the failure message too)."""
    if dtype is None:
        dtype = got.dtype
    if dtype not in HALF_ATOL:
        raise TypeError(f"assert_half expects bf16 / fp16, got {dtype}")
    if isinstance(got, torch.Tensor):
        got = got.detach().double().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    atol = HALF_ATOL[dtype]
    err = np.abs(got - ref)
    large = np.abs(ref) >= LARGE
    n_large = int(large.sum())
    small_err = float(err[~large].max(initial=0.0))
    bound = np.where(large, half_ulp(ref, dtype) + atol, atol)
    worst = float((err - bound).max(initial=-1.0))
    large_err = float(err[large].max(initial=0.0))
    assert worst <= 0, (f"{what}: {dtype} error above the parity bound by {worst:.3e} "
                        f"(max |err| {small_err:.3e} where |ref| < 8 against {atol:g}; "
                        f"{n_large} elements with |ref| >= 8, max |err| {large_err:.3e} there)")
    return n_large
