"""Width-read and mix + depth-write for a backbone of m blocks: the two halves
of a hyper-connection layer around its wrapped module.

    u  = hc_read(R, x)                   u[t,k,:]  = sum_j R[t,k,j] x[t,j,:]
    x' = hc_mix_write(H, x, W, f, v)     x'[t,i,:] = sum_j H_ij x_j
                                                     [+ (v_i - (H v)_i) v^T x]
                                                     + sum_k W_ik f_k

``hc_read`` replaces the read einsum ``einsum(read_in, x, "b m n, b n d ->
b m d")`` (hyperconnections/cghc.py:410; ghc.py:116, mhc.py:138,
attnhc.py:154). ``hc_mix_write`` replaces the write einsum
(cghc.py:417, ``"b n m, b m d -> b n d"``) followed by ``stream_mix_add``
(cghc.py:449), without materialising the written term in HBM; ``v`` is the
projection direction of the projected mix (cghc.py:341-350).

Shapes: x [*, n, D]; R [*, m, n]; H [*, n, n]; W [*, n, m]; f [*, m, D];
v [*, n], or [n] / [1, n] broadcast over the tokens. 1 <= m <= 4, n <= 8.
x and f share one stream dtype (float32, float16 or bfloat16); the weights
are computed in float32 and their gradients are returned in their own dtype.
"""

from __future__ import annotations

import math

import torch

from .. import _lib
from .stream_mix import MAX_STREAMS

MAX_WIDTH = 4


def _require_cuda(name: str, tensors) -> None:
    if not _lib.available():
        raise RuntimeError(f"{name} requires the hyperconnections_b200 CUDA kernels (libhcops.so)")
    for tname, t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name} requires CUDA tensors ({tname} is on {t.device})")


def _f32(t: torch.Tensor, shape) -> torch.Tensor:
    return t.to(torch.float32).contiguous().view(*shape)


class _ReadFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, R, x):
        lead = x.shape[:-2]
        n, D = x.shape[-2], x.shape[-1]
        m = R.shape[-2]
        T = math.prod(lead)
        x_c = x.contiguous().view(T, n, D)
        R_c = _f32(R, (T, m, n))
        u = torch.empty(T, m, D, dtype=x.dtype, device=x.device)
        with _lib.on_device(x_c):
            rc = _lib.lib().hc_read_fwd(R_c.data_ptr(), x_c.data_ptr(), u.data_ptr(), T, n, m, D,
                                        _lib.dtype_code(x.dtype), _lib.stream_of(x_c))
        _lib.check(rc, "hc_read_fwd")
        ctx.save_for_backward(R_c, x_c)
        ctx.lead, ctx.R_dtype = lead, R.dtype
        return u.view(*lead, m, D)

    @staticmethod
    def backward(ctx, g_u):
        R_c, x_c = ctx.saved_tensors
        T, n, D = x_c.shape
        m = R_c.shape[1]
        need_R, need_x = ctx.needs_input_grad
        dt, dev = x_c.dtype, x_c.device
        g = g_u.to(dt).contiguous().view(T, m, D)
        grad_x = torch.empty_like(x_c) if need_x else None
        grad_R = torch.empty(T, m, n, dtype=torch.float32, device=dev) if need_R else None
        with _lib.on_device(x_c):
            rc = _lib.lib().hc_read_bwd(g.data_ptr(), R_c.data_ptr(), x_c.data_ptr(), _lib.ptr(grad_x),
                                        _lib.ptr(grad_R), T, n, m, D, _lib.dtype_code(dt), _lib.stream_of(x_c))
        _lib.check(rc, "hc_read_bwd")
        lead = ctx.lead
        return (grad_R.view(*lead, m, n).to(ctx.R_dtype) if need_R else None,
                grad_x.view(*lead, n, D) if need_x else None)


class _MixWriteFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, H, x, W, f, v):
        lead = x.shape[:-2]
        n, D = x.shape[-2], x.shape[-1]
        m = W.shape[-1]
        T = math.prod(lead)
        x_c = x.contiguous().view(T, n, D)
        f_c = f.to(x.dtype).contiguous().view(T, m, D)
        H_c = _f32(H, (T, n, n))
        W_c = _f32(W, (T, n, m))
        v_c = None if v is None else _f32(v.expand(*lead, n), (T, n))
        out = torch.empty_like(x_c)
        with _lib.on_device(x_c):
            rc = _lib.lib().hc_mix_write_fwd(H_c.data_ptr(), x_c.data_ptr(), W_c.data_ptr(), f_c.data_ptr(),
                                             _lib.ptr(v_c), out.data_ptr(), T, n, m, D,
                                             _lib.dtype_code(x.dtype), _lib.stream_of(x_c))
        _lib.check(rc, "hc_mix_write_fwd")
        ctx.save_for_backward(H_c, x_c, W_c, f_c, v_c)
        ctx.lead = lead
        ctx.dtypes = (H.dtype, W.dtype, f.dtype, None if v is None else v.dtype)
        ctx.v_shape = None if v is None else v.shape
        return out.view(*lead, n, D)

    @staticmethod
    def backward(ctx, g):
        H_c, x_c, W_c, f_c, v_c = ctx.saved_tensors
        T, n, D = x_c.shape
        m = W_c.shape[2]
        need_H, need_x, need_W, need_f, need_v = ctx.needs_input_grad
        need_v = need_v and v_c is not None
        dt, dev = x_c.dtype, x_c.device
        g_c = g.to(dt).contiguous().view(T, n, D)
        grad_x = torch.empty_like(x_c) if need_x else None
        grad_f = torch.empty(T, m, D, dtype=dt, device=dev) if need_f else None
        grad_H = torch.empty(T, n, n, dtype=torch.float32, device=dev) if need_H else None
        grad_W = torch.empty(T, n, m, dtype=torch.float32, device=dev) if need_W else None
        grad_v = torch.empty(T, n, dtype=torch.float32, device=dev) if need_v else None
        with _lib.on_device(x_c):
            rc = _lib.lib().hc_mix_write_bwd(
                g_c.data_ptr(), H_c.data_ptr(), x_c.data_ptr(), W_c.data_ptr(), f_c.data_ptr(), _lib.ptr(v_c),
                _lib.ptr(grad_x), _lib.ptr(grad_f), _lib.ptr(grad_H), _lib.ptr(grad_W), _lib.ptr(grad_v),
                T, n, m, D, _lib.dtype_code(dt), _lib.stream_of(x_c))
        _lib.check(rc, "hc_mix_write_bwd")
        lead = ctx.lead
        H_dt, W_dt, f_dt, v_dt = ctx.dtypes
        gv = None
        if need_v:
            gv = grad_v.view(*lead, n)
            # a direction broadcast over the tokens gets the sum of the per-token gradients
            vs = ctx.v_shape
            extra = gv.dim() - len(vs)
            gv = gv.sum(dim=tuple(range(extra))) if extra > 0 else gv
            keep = tuple(i for i, s in enumerate(vs) if s == 1 and gv.shape[i] != 1)
            if keep:
                gv = gv.sum(dim=keep, keepdim=True)
            gv = gv.to(v_dt)
        return (grad_H.view(*lead, n, n).to(H_dt) if need_H else None,
                grad_x.view(*lead, n, D) if need_x else None,
                grad_W.view(*lead, n, m).to(W_dt) if need_W else None,
                grad_f.view(*lead, m, D).to(f_dt) if need_f else None,
                gv)


def _check_width(name: str, n: int, m: int) -> None:
    if n > MAX_STREAMS:
        raise RuntimeError(f"{name} supports n <= {MAX_STREAMS} streams, got n={n}")
    if not 1 <= m <= MAX_WIDTH:
        raise RuntimeError(f"{name} supports 1 <= m <= {MAX_WIDTH} backbone blocks, got m={m}")


def hc_read(R: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """u = R x per token: R [*, m, n], x [*, n, D] -> u [*, m, D] (see module doc)."""
    _require_cuda("hc_read", (("R", R), ("x", x)))
    if x.dim() < 2:
        raise ValueError("x must be [*, n, D]")
    n, D = x.shape[-2], x.shape[-1]
    lead = x.shape[:-2]
    assert R.dim() == x.dim() and R.shape[:-2] == lead and R.shape[-1] == n, (
        f"R must be {(*lead, 'm', n)}, got {tuple(R.shape)}")
    _check_width("hc_read", n, R.shape[-2])
    return _ReadFn.apply(R, x)


def hc_mix_write(H: torch.Tensor, x: torch.Tensor, W: torch.Tensor, f: torch.Tensor, v=None) -> torch.Tensor:
    """x' = H x [+ projection] + W f per token (see module doc)."""
    _require_cuda("hc_mix_write", (("H", H), ("x", x), ("W", W), ("f", f), ("v", v)))
    if x.dim() < 2:
        raise ValueError("x must be [*, n, D]")
    n, D = x.shape[-2], x.shape[-1]
    lead = x.shape[:-2]
    m = W.shape[-1]
    assert H.shape == (*lead, n, n), f"H must be {(*lead, n, n)}, got {tuple(H.shape)}"
    assert W.shape == (*lead, n, m), f"W must be {(*lead, n, 'm')}, got {tuple(W.shape)}"
    assert f.shape == (*lead, m, D), f"f must be {(*lead, m, D)}, got {tuple(f.shape)}"
    if v is not None:
        assert v.shape[-1] == n and v.dim() <= len(lead) + 1, f"v must broadcast to {(*lead, n)}"
        torch.broadcast_shapes(v.shape, (*lead, n))
    _check_width("hc_mix_write", n, m)
    return _MixWriteFn.apply(H, x, W, f, v)
