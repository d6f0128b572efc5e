"""Fused stream mixing, drop-in for ``hyperconnections.ops.stream_mix``.

Computes  out = Phi @ x + Y                              [no-proj]
or        out = Phi @ x + (v - Phi@v)(v^T x) + Y        [proj]

with Phi [B,N,N], x/Y [B,N,D], v [B,N]. Same signature, shape asserts, error
messages and dtype conventions as the reference
(hyperconnections/ops/stream_mix.py:57-86 and
ops/stream_mix_small_nb.py:326-414):

* fp32 accumulation; the output has x's dtype;
* grad_Phi is produced in fp32 and cast to Phi's dtype, grad_x has x's dtype,
  grad_Y is grad_out itself, grad_v is fp32 cast to v's dtype and only
  produced when v requires it (stream_mix_small_nb.py:379-391);
* CPU tensors raise RuntimeError("... requires CUDA tensors").

One forward kernel and one backward kernel (hc_stream_mix_fwd/bwd) replace the
reference's small-NB / big-NB Triton pair: the backward reads grad_out and x
once and produces grad_x, grad_Phi and grad_v together, so there is no
size-based dispatch (the reference's A100 L2 heuristic,
stream_mix.py:45-54, has no counterpart).
"""

from __future__ import annotations

import torch

from .. import _lib

HAS_TRITON = _lib.available()
"""Name kept from the reference (ops/__init__.py:1); here it means that the
sm_100a kernels of libhcops.so are available."""

MAX_STREAMS = 8       # the fused step and the m-block read / mix-write
MAX_STREAMS_ADD = 32  # stream_mix_add: n <= 8 register kernels, 9..32 shared-memory kernels


def _param_dtype(Phi: torch.Tensor, v: torch.Tensor | None, x: torch.Tensor) -> torch.dtype:
    """Phi and v travel in x's dtype when they already have it, else in fp32
    (every conversion to fp32 is exact)."""
    if Phi.dtype == x.dtype and (v is None or v.dtype == x.dtype):
        return x.dtype
    return torch.float32


class _StreamMixFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Phi, x, Y, v):
        x_c = x.contiguous()
        pdt = _param_dtype(Phi, v, x)
        Phi_c = Phi.to(pdt).contiguous()
        Y_c = Y.to(x.dtype).contiguous()
        v_c = v.to(pdt).contiguous() if v is not None else None
        B, N, D = x_c.shape
        out = torch.empty_like(x_c)
        lib = _lib.lib()
        with _lib.on_device(x_c):
            rc = lib.hc_stream_mix_fwd(
                Phi_c.data_ptr(), x_c.data_ptr(), Y_c.data_ptr(), _lib.ptr(v_c), out.data_ptr(),
                B, N, D, _lib.dtype_code(x_c.dtype), _lib.dtype_code(pdt), _lib.stream_of(x_c),
            )
        _lib.check(rc, "hc_stream_mix_fwd")
        ctx.save_for_backward(Phi_c, x_c, v_c)
        ctx.phi_dtype = Phi.dtype
        ctx.v_dtype = v.dtype if v is not None else None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        Phi_c, x_c, v_c = ctx.saved_tensors
        B, N, D = x_c.shape
        G = grad_out.to(x_c.dtype).contiguous()
        need_phi, need_x, need_y, need_v = ctx.needs_input_grad
        need_v = need_v and v_c is not None
        grad_x = torch.empty_like(x_c) if need_x else None
        grad_phi = torch.empty(B, N, N, dtype=torch.float32, device=x_c.device) if need_phi else None
        grad_v = torch.empty(B, N, dtype=torch.float32, device=x_c.device) if need_v else None
        if need_x or need_phi or need_v:
            lib = _lib.lib()
            with _lib.on_device(x_c):
                rc = lib.hc_stream_mix_bwd(
                    G.data_ptr(), Phi_c.data_ptr(), x_c.data_ptr(), _lib.ptr(v_c),
                    _lib.ptr(grad_x), _lib.ptr(grad_phi), _lib.ptr(grad_v),
                    B, N, D, _lib.dtype_code(x_c.dtype), _lib.dtype_code(Phi_c.dtype), _lib.stream_of(x_c),
                )
            _lib.check(rc, "hc_stream_mix_bwd")
        return (
            grad_phi.to(ctx.phi_dtype) if need_phi else None,
            grad_x,
            grad_out if need_y else None,
            grad_v.to(ctx.v_dtype) if need_v else None,
        )


def stream_mix_add(
    Phi: torch.Tensor,
    x: torch.Tensor,
    Y: torch.Tensor,
    v: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused  out = Phi @ x + Y  (or projected variant).

    Args:
        Phi: [B, N, N] transition matrix.
        x:   [B, N, D] stream state.
        Y:   [B, N, D] source term.
        v:   [B, N]    unit-norm projection direction, or None.

    Returns:
        out: [B, N, D], dtype of x.
    """
    if not HAS_TRITON:
        raise RuntimeError("stream_mix_add requires the hyperconnections_b200 CUDA kernels (libhcops.so)")
    if not x.is_cuda:
        raise RuntimeError("stream_mix_add requires CUDA tensors")
    B, N, D = x.shape
    assert Phi.shape == (B, N, N)
    assert Y.shape == (B, N, D)
    if v is not None:
        assert v.shape == (B, N)
    if not (Phi.is_cuda and Y.is_cuda and (v is None or v.is_cuda)):
        raise RuntimeError("stream_mix_add requires CUDA tensors")
    if N > MAX_STREAMS_ADD:
        raise RuntimeError(f"stream_mix_add supports N <= {MAX_STREAMS_ADD} streams, got N={N}")
    return _StreamMixFn.apply(Phi, x, Y, v)
