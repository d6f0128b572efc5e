"""CGHC's generator A per token (hyperconnections/cghc.py:219-315), assembled
by one kernel from the module's pre-activations, forward and backward; and
CGHC's transition Phi = exp(A) (cghc.py:317-321) in one kernel per direction,
the generator fused with the Pade [7/7] exponential.

    A = cghc_generator(M=..., logit_conserv=..., R=..., diag_pre=..., scores=...,
                       logit_diss=..., dt_range_conserv=(lo, hi),
                       dt_range_diss=(lo, hi), vec_dt=False)

The pre-activations are what the reference's Linear layers and static
parameters give (one add each): M = conserv_A + conv_pred(x), R = diss_A +
diss_pred(x), diag_pre = diss_diag + diss_pred(x), scores = laplacian_A +
laplacian_pred(x), logit_conserv = log_dt_conserv + dt_proj_conserv(x),
logit_diss = log_dt_diss + dt_proj_diss(x). Pass the ones the generator type
uses: conservative (M, logit_conserv), PSD dissipation (R), diagonal
dissipation (diag_pre), Laplacian dissipation (scores), any dissipation also
logit_diss. Shapes [*, n, n] / [*, n] / [*, n_dt] with n_dt = n if vec_dt else
1, n <= 8; computed in float32, A returned as [*, n, n] float32.

With ``matrix_exp`` and the read / mix-write kernels this makes CGHC's
generator -> transition -> mix chain a short sequence of launches instead of
the reference's tens of small elementwise ops per layer.
"""

from __future__ import annotations

import math

import torch

from .. import _lib

_CONSERV, _PSD, _DIAG, _LAP = 1, 2, 4, 8


class _GeneratorFn(torch.autograd.Function):
    """A = generator(pre-activations); with fused=True, Phi = exp(A) instead
    (hc_cghc_transition_fwd/bwd), the upstream gradient being dL/dPhi."""

    @staticmethod
    def forward(ctx, M, lc, R, dpre, S, ld, n, T, vec_dt, flags, ranges, fused):
        f32 = lambda t, *shape: None if t is None else t.to(torch.float32).contiguous().view(*shape)  # noqa: E731
        nd = n if vec_dt else 1
        ins = [f32(M, T, n, n), f32(lc, T, nd), f32(R, T, n, n), f32(dpre, T, n), f32(S, T, n, n), f32(ld, T, nd)]
        dev = next(t.device for t in ins if t is not None)
        A = torch.empty(T, n, n, dtype=torch.float32, device=dev)
        name = "hc_cghc_transition_fwd" if fused else "hc_cghc_generator_fwd"
        with _lib.on_device(A):
            rc = getattr(_lib.lib(), name)(*[_lib.ptr(t) for t in ins], A.data_ptr(), T, n, int(vec_dt), flags,
                                           *ranges, _lib.stream_of(A))
        _lib.check(rc, name)
        ctx.fused = fused
        ctx.save_for_backward(*[t if t is not None else torch.empty(0) for t in ins])
        ctx.present = [t is not None for t in ins]
        ctx.meta = (n, T, vec_dt, flags, ranges)
        ctx.dtypes = [None if t is None else t.dtype for t in (M, lc, R, dpre, S, ld)]
        ctx.shapes = [None if t is None else t.shape for t in (M, lc, R, dpre, S, ld)]
        return A

    @staticmethod
    def backward(ctx, G):
        saved = ctx.saved_tensors
        ins = [t if p else None for t, p in zip(saved, ctx.present)]
        n, T, vec_dt, flags, ranges = ctx.meta
        need = ctx.needs_input_grad[:6]
        outs = [torch.empty_like(t) if (t is not None and nd) else None for t, nd in zip(ins, need)]
        Gc = G.to(torch.float32).contiguous().view(T, n, n)
        name = "hc_cghc_transition_bwd" if ctx.fused else "hc_cghc_generator_bwd"
        with _lib.on_device(Gc):
            rc = getattr(_lib.lib(), name)(
                *[_lib.ptr(t) for t in ins], Gc.data_ptr(),
                # kernel order of the gradients: dM, dlc, dR, ddpre, dS, dld
                *[_lib.ptr(t) for t in outs], T, n, int(vec_dt), flags, *ranges, _lib.stream_of(Gc))
        _lib.check(rc, name)
        grads = [None if g is None else g.view(shape).to(dt)
                 for g, shape, dt in zip(outs, ctx.shapes, ctx.dtypes)]
        return (*grads, None, None, None, None, None, None)


def cghc_generator(*, M=None, logit_conserv=None, R=None, diag_pre=None, scores=None, logit_diss=None,
                   dt_range_conserv=(0.001, 1.0), dt_range_diss=(0.001, 1.0), vec_dt: bool = False):
    """Generator A [*, n, n] of CGHC from its pre-activations (see module doc)."""
    return _apply(M, logit_conserv, R, diag_pre, scores, logit_diss, dt_range_conserv, dt_range_diss, vec_dt, False)


def cghc_transition(*, M=None, logit_conserv=None, R=None, diag_pre=None, scores=None, logit_diss=None,
                    dt_range_conserv=(0.001, 1.0), dt_range_diss=(0.001, 1.0), vec_dt: bool = False):
    """CGHC's transition Phi = exp(A) [*, n, n] (cghc.py:317-321, with
    matrix_exp's Pade [7/7]) straight from the pre-activations, one kernel per
    direction; the same values as ``matrix_exp(cghc_generator(...))``."""
    return _apply(M, logit_conserv, R, diag_pre, scores, logit_diss, dt_range_conserv, dt_range_diss, vec_dt, True)


def _apply(M, logit_conserv, R, diag_pre, scores, logit_diss, dt_range_conserv, dt_range_diss, vec_dt, fused):
    if not _lib.available():
        raise RuntimeError("cghc_generator requires the hyperconnections_b200 CUDA kernels (libhcops.so)")
    flags = (_CONSERV if M is not None else 0) | (_PSD if R is not None else 0) | \
        (_DIAG if diag_pre is not None else 0) | (_LAP if scores is not None else 0)
    if flags == 0:
        raise ValueError("cghc_generator needs at least one of M, R, diag_pre, scores")
    if M is not None and logit_conserv is None:
        raise ValueError("the conservative term needs logit_conserv")
    if flags & (_PSD | _DIAG | _LAP) and logit_diss is None:
        raise ValueError("a dissipative term needs logit_diss")
    ref = next(t for t in (M, R, scores, diag_pre) if t is not None)
    for t in (M, logit_conserv, R, diag_pre, scores, logit_diss):
        if t is not None and not t.is_cuda:
            raise RuntimeError("cghc_generator requires CUDA tensors")
    n = ref.shape[-1]
    lead = ref.shape[:-2] if ref is not diag_pre else ref.shape[:-1]
    if not 1 <= n <= 8:
        raise RuntimeError(f"cghc_generator supports 1 <= n <= 8, got n={n}")
    T = math.prod(lead)
    ranges = (float(dt_range_conserv[0]), float(dt_range_conserv[1]), float(dt_range_diss[0]),
              float(dt_range_diss[1]))
    A = _GeneratorFn.apply(M, logit_conserv, R, diag_pre, scores, logit_diss, n, T, bool(vec_dt), flags, ranges,
                           fused)
    return A.view(*lead, n, n)
