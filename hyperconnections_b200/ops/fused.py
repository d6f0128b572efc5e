"""The fused hyper-connection step with one backbone block (m = 1).

    u       = sum_j alpha_j x_j                 (width-read,  cghc.py:410)
    x_out_i = sum_j H_ij x_j + beta_i f         (residual mix + depth-write,
                                                 cghc.py:417 and :449)

The reference computes this as three separate operations (two einsums and
stream_mix_add) and materialises the write-out Y = beta f in HBM. Here one
forward kernel reads x and f once and writes u and x_out once; one backward
kernel reads the two upstream gradients, x and f once and writes grad_x,
grad_f and the per-token parameter gradients grad_H, grad_alpha, grad_beta.

Shapes: x [*, n, D]; f [*, D]; H [*, n, n]; alpha, beta [*, n], where * is
any number of leading token dimensions. x and f share one stream dtype
(float32, float16 or bfloat16); H, alpha and beta are float32 (other dtypes are
converted). Returns (u [*, D], x_out [*, n, D]) in the stream dtype.
"""

from __future__ import annotations

import torch

from .. import _lib
from .stream_mix import MAX_STREAMS


class _FusedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, f, H, alpha, beta):
        lead = x.shape[:-2]
        n, D = x.shape[-2], x.shape[-1]
        x_c = x.contiguous().view(-1, n, D)
        T = x_c.shape[0]
        f_c = f.to(x.dtype).contiguous().view(T, D)
        H_c = H.to(torch.float32).contiguous().view(T, n, n)
        a_c = alpha.to(torch.float32).contiguous().view(T, n)
        b_c = beta.to(torch.float32).contiguous().view(T, n)
        u = torch.empty(T, D, dtype=x.dtype, device=x.device)
        x_out = torch.empty_like(x_c)
        lib = _lib.lib()
        with _lib.on_device(x_c):
            rc = lib.hc_fused_fwd(
                x_c.data_ptr(), f_c.data_ptr(), H_c.data_ptr(), a_c.data_ptr(), b_c.data_ptr(),
                u.data_ptr(), x_out.data_ptr(), T, n, D, _lib.dtype_code(x.dtype), _lib.stream_of(x_c),
            )
        _lib.check(rc, "hc_fused_fwd")
        ctx.save_for_backward(x_c, f_c, H_c, a_c, b_c)
        ctx.lead = lead
        ctx.dtypes = (f.dtype, H.dtype, alpha.dtype, beta.dtype)
        return u.view(*lead, D), x_out.view(*lead, n, D)

    @staticmethod
    def backward(ctx, g_u, g_x):
        x_c, f_c, H_c, a_c, b_c = ctx.saved_tensors
        T, n, D = x_c.shape
        need_x, need_f, need_H, need_a, need_b = ctx.needs_input_grad
        dt = x_c.dtype
        g_u = torch.zeros(T, D, dtype=dt, device=x_c.device) if g_u is None else g_u.to(dt).contiguous().view(T, D)
        g_x = torch.zeros(T, n, D, dtype=dt, device=x_c.device) if g_x is None else g_x.to(dt).contiguous().view(T, n, D)
        dev = x_c.device
        grad_x = torch.empty_like(x_c) if need_x else None
        grad_f = torch.empty(T, D, dtype=dt, device=dev) if need_f else None
        grad_H = torch.empty(T, n, n, dtype=torch.float32, device=dev) if need_H else None
        grad_a = torch.empty(T, n, dtype=torch.float32, device=dev) if need_a else None
        grad_b = torch.empty(T, n, dtype=torch.float32, device=dev) if need_b else None
        lib = _lib.lib()
        with _lib.on_device(x_c):
            rc = lib.hc_fused_bwd(
                g_u.data_ptr(), g_x.data_ptr(), x_c.data_ptr(), f_c.data_ptr(), H_c.data_ptr(),
                a_c.data_ptr(), b_c.data_ptr(), _lib.ptr(grad_x), _lib.ptr(grad_f), _lib.ptr(grad_H),
                _lib.ptr(grad_a), _lib.ptr(grad_b), T, n, D, _lib.dtype_code(dt), _lib.stream_of(x_c),
            )
        _lib.check(rc, "hc_fused_bwd")
        lead = ctx.lead
        f_dt, H_dt, a_dt, b_dt = ctx.dtypes
        return (
            grad_x.view(*lead, n, D) if need_x else None,
            grad_f.view(*lead, D).to(f_dt) if need_f else None,
            grad_H.view(*lead, n, n).to(H_dt) if need_H else None,
            grad_a.view(*lead, n).to(a_dt) if need_a else None,
            grad_b.view(*lead, n).to(b_dt) if need_b else None,
        )


def stream_mix_fused(
    x: torch.Tensor,
    f: torch.Tensor,
    H: torch.Tensor,
    alpha: torch.Tensor,
    beta: torch.Tensor,
):
    """(u, x_out) = (sum_j alpha_j x_j, H x + beta f) per token; see module doc."""
    if not _lib.available():
        raise RuntimeError("stream_mix_fused requires the hyperconnections_b200 CUDA kernels (libhcops.so)")
    for name, t in (("x", x), ("f", f), ("H", H), ("alpha", alpha), ("beta", beta)):
        if not t.is_cuda:
            raise RuntimeError(f"stream_mix_fused requires CUDA tensors ({name} is on {t.device})")
    if x.dim() < 2:
        raise ValueError("x must be [*, n, D]")
    n, D = x.shape[-2], x.shape[-1]
    lead = x.shape[:-2]
    if n > MAX_STREAMS:
        raise RuntimeError(f"stream_mix_fused supports n <= {MAX_STREAMS} streams, got n={n}")
    assert f.shape == (*lead, D), f"f must be {(*lead, D)}, got {tuple(f.shape)}"
    assert H.shape == (*lead, n, n), f"H must be {(*lead, n, n)}, got {tuple(H.shape)}"
    assert alpha.shape == (*lead, n), f"alpha must be {(*lead, n)}, got {tuple(alpha.shape)}"
    assert beta.shape == (*lead, n), f"beta must be {(*lead, n)}, got {tuple(beta.shape)}"
    return _FusedFn.apply(x, f, H, alpha, beta)
