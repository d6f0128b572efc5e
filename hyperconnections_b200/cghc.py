"""CGHC layer on the B200 kernels: drop-in for the reference's
``hyperconnections.cghc.ContinuousGenHyperConnections`` (cghc.py:14-457).

Same constructor arguments, parameters, buffers and ``state_dict`` keys as the
reference, so a reference layer's weights load unchanged, and the same
forward semantics (cghc.py:394-457): ``x [*, n * block]`` -> ``[*, n * block]``.
The forward runs

    x_norm  = RMSNorm(x)                           once (cghc.py:222, :326, :346)
    h       = one GEMM of x_norm against every Linear head of the layer
    R, W    = sigmoid read / 2 sigmoid write weights          (cghc.py:323-339)
    u       = hc_read(R, x)                        width-read (cghc.py:410)
    f       = module(u)                                        (cghc.py:413)
    Phi     = cghc_transition(pre-activations)     one kernel: the generator
                                                   (cghc.py:219-315) fused with
                                                   the Pade exponential (:321)
    x_new   = hc_mix_write(Phi, x, W, f, v)        depth-write + mix (cghc.py:417, :449)

so the written term Y = W f is never materialised, the generator's tens of
small elementwise ops and the exponential are one launch, and the Linear heads that read the
normalised stream (read, write, two dt heads, generator heads, projection) are
one GEMM instead of six reads of x_norm.

Deliberate differences, all within the parity tolerances: Phi stays float32
(the reference casts it to the stream dtype, cghc.py:321); the heads' outputs
are taken to float32 before the nonlinearities; ``use_triton`` is accepted and
ignored (there is no other backend).
"""

from __future__ import annotations

import math
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import cghc_transition, hc_mix_write, hc_read

GeneratorType = Literal["conservative", "psd_diss", "diagonal_diss", "laplacian", "conservative_diag_diss",
                        "conservative_psd_diss", "conservative_laplacian"]

_CONSERV = {"conservative", "conservative_diag_diss", "conservative_psd_diss", "conservative_laplacian"}
_PSD = {"psd_diss", "conservative_psd_diss"}
_DIAG = {"diagonal_diss", "conservative_diag_diss"}
_LAPLACIAN = {"laplacian", "conservative_laplacian"}


def _logit_of_dt(dt: float, lo: float, hi: float) -> float:
    """Pre-activation whose sigmoid maps to dt in (lo, hi)."""
    p = min(max((dt - lo) / (hi - lo), 1e-4), 1 - 1e-4)
    return math.log(p / (1 - p))


class ContinuousGenHyperConnections(nn.Module):
    """Continuous generalised hyper-connection layer (see module doc).

    Args are the reference's (cghc.py:15-40): n streams, m backbone blocks,
    input_dim = n / m * embed_dim, the wrapped module, the generator type,
    projection ("mean" / "v" / "none"), dt and its range, learn_dt, bias of
    the read / write heads, elementwise_affine of the RMSNorm, vec_dt.
    """

    def __init__(self, n: int, m: int, input_dim: int, embed_dim: int, module: nn.Module, dt: float = 0.01,
                 generator_type: GeneratorType = "conservative_psd_diss",
                 projection: Literal["mean", "v", "none"] = "none", learn_dt: bool = False, dt_min: float = 0.001,
                 dt_max: float = 1.0, bias: bool = False, elementwise_affine: bool = False, use_triton: bool = True,
                 vec_dt: bool = False):
        super().__init__()
        if embed_dim % m:
            raise ValueError(f"embed_dim ({embed_dim}) must be divisible by m ({m})")
        if input_dim != n * embed_dim // m or (n * embed_dim) % m:
            raise ValueError(f"input_dim must be (n/m)*embed_dim = {n * embed_dim // m}, got {input_dim}")
        if not dt_min < dt < dt_max:
            raise ValueError(f"dt ({dt}) must lie strictly in (dt_min, dt_max) = ({dt_min}, {dt_max})")
        if generator_type not in _CONSERV | _PSD | _DIAG | _LAPLACIAN:
            raise ValueError(f"unknown generator_type {generator_type!r}")
        self.n, self.m, self.input_dim, self.embed_dim = n, m, input_dim, embed_dim
        self.block_size = embed_dim // m
        self.generator_type, self.projection, self.vec_dt = generator_type, projection, vec_dt
        self.dt_min_cons = self.dt_min_diss = dt_min
        self.dt_max_cons = self.dt_max_diss = dt_max
        self.log_dt_init_cons = self.log_dt_init_diss = math.log(dt)
        n_dt = n if vec_dt else 1

        self.read_in = nn.Parameter(torch.empty(n, m))
        self.alpha_read_in = nn.Parameter(torch.empty(1))
        self.write_out = nn.Parameter(torch.empty(n, m))
        self.alpha_write_out = nn.Parameter(torch.empty(1))
        self.proj_read_in = nn.Linear(input_dim, n * m, bias=bias)
        self.proj_write_out = nn.Linear(input_dim, n * m, bias=bias)
        self.log_dt_conserv = nn.Parameter(torch.empty(n_dt), requires_grad=learn_dt)
        self.log_dt_diss = nn.Parameter(torch.empty(n_dt), requires_grad=learn_dt)
        self.dt_proj_conserv = nn.Linear(input_dim, n_dt, bias=True)
        self.dt_proj_diss = nn.Linear(input_dim, n_dt, bias=True)
        if generator_type in _CONSERV:
            self.conserv_A = nn.Parameter(torch.eye(n))
            self.conv_pred = nn.Linear(input_dim, n * n, bias=True)
        if generator_type in _PSD:
            self.diss_A = nn.Parameter(torch.zeros(n, n))
            self.diss_pred = nn.Linear(input_dim, n * n, bias=True)
        if generator_type in _DIAG:
            self.diss_diag = nn.Parameter(torch.full((n,), -2.0))
            self.diss_pred = nn.Linear(input_dim, n, bias=True)
        if generator_type in _LAPLACIAN:
            self.laplacian_A = nn.Parameter(torch.zeros(n, n))
            self.laplacian_pred = nn.Linear(input_dim, n * n, bias=True)
        if projection == "mean":
            self.register_buffer("projection_dir", torch.ones(n) / math.sqrt(n))
        elif projection == "v":
            self.projection_dir = nn.Linear(input_dim, n, bias=True)
        elif projection == "none":
            self.projection_dir = None
        else:
            raise ValueError(f"unknown projection {projection!r}")
        self.norm = nn.RMSNorm(input_dim, elementwise_affine=elementwise_affine)
        self.module = module
        self.init_weights()

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_weights(self):
        """The reference's initial distribution (cghc.py:130-217): read
        weights at sigmoid^-1(1/n) with 1% noise, write weights near 2
        sigmoid(0) = 1, static generator near I (conservative) / 0, dt at its
        initial value, every Linear head with std-0.01 weights and zero bias."""
        n = self.n
        tn = lambda t: nn.init.trunc_normal_(t, std=0.01)  # noqa: E731
        self.read_in.fill_(math.log(1.0 / (n - 1)) if n > 1 else 10.0).add_(0.01 * torch.randn_like(self.read_in))
        tn(self.write_out)
        self.alpha_read_in.fill_(0.01)
        self.alpha_write_out.fill_(0.01)
        if hasattr(self, "conserv_A"):
            self.conserv_A.copy_(torch.eye(n)).add_(tn(torch.empty(n, n)))
        if hasattr(self, "diss_A"):
            tn(self.diss_A)
        if hasattr(self, "diss_diag"):
            self.diss_diag.fill_(-2.0)
        if hasattr(self, "laplacian_A"):
            self.laplacian_A.fill_(-2.0)
        for head in self._generator_heads() + [self.dt_proj_conserv, self.dt_proj_diss, self.proj_read_in,
                                               self.proj_write_out]:
            tn(head.weight)
            if head.bias is not None:
                head.bias.zero_()
        self.log_dt_conserv.fill_(_logit_of_dt(math.exp(self.log_dt_init_cons), self.dt_min_cons, self.dt_max_cons))
        self.log_dt_diss.fill_(_logit_of_dt(math.exp(self.log_dt_init_diss), self.dt_min_diss, self.dt_max_diss))
        if self.projection == "mean":
            d = torch.full((n,), 1.0 / math.sqrt(n)) + 0.01 * torch.randn(n)
            self.projection_dir.copy_(d / d.norm())
        elif self.projection == "v":
            tn(self.projection_dir.weight)
            self.projection_dir.bias.fill_(1.0 / math.sqrt(n))
        if self.norm.weight is not None:
            self.norm.weight.fill_(1.0)

    def _generator_heads(self) -> list:
        return [getattr(self, k) for k in ("conv_pred", "diss_pred", "laplacian_pred") if hasattr(self, k)]

    # --------------------------------------------------------------- forward
    def _heads(self):
        """(name, Linear, width) of every head that reads the normalised stream
        and that the generator type uses (an unused head gets no gradient, as
        in the reference)."""
        n, m, gt = self.n, self.m, self.generator_type
        heads = [("read", self.proj_read_in, n * m), ("write", self.proj_write_out, n * m)]
        if gt in _CONSERV:
            heads.append(("dtc", self.dt_proj_conserv, self.dt_proj_conserv.out_features))
        if gt in _PSD | _DIAG | _LAPLACIAN:
            heads.append(("dtd", self.dt_proj_diss, self.dt_proj_diss.out_features))
        for name in ("conv_pred", "diss_pred", "laplacian_pred"):
            if hasattr(self, name):
                lin = getattr(self, name)
                heads.append((name, lin, lin.out_features))
        if self.projection == "v":
            heads.append(("v", self.projection_dir, n))
        return heads

    def forward(self, x: torch.Tensor, **kwargs) -> torch.Tensor:
        n, m, blk = self.n, self.m, self.block_size
        lead = x.shape[:-1]
        xs = x.reshape(-1, n, blk)
        T = xs.shape[0]
        xn = self.norm(xs.reshape(T, n * blk))
        heads = self._heads()
        weight = torch.cat([lin.weight for _, lin, _ in heads])
        bias = torch.cat([lin.bias if lin.bias is not None else lin.weight.new_zeros(w) for _, lin, w in heads])
        h = dict(zip([k for k, _, _ in heads], F.linear(xn, weight, bias).float().split([w for *_, w in heads], -1)))

        read = torch.sigmoid(self.alpha_read_in * h["read"].view(T, n, m) + self.read_in).transpose(1, 2)
        write = 2.0 * torch.sigmoid(self.alpha_write_out * h["write"].view(T, n, m) + self.write_out)
        u = hc_read(read, xs)
        f = self.module(u.reshape(*lead, self.embed_dim), **kwargs).reshape(T, m, blk)

        gt = self.generator_type
        dissipative = gt in _PSD | _DIAG | _LAPLACIAN
        Phi = cghc_transition(
            M=self.conserv_A + h["conv_pred"].view(T, n, n) if gt in _CONSERV else None,
            logit_conserv=self.log_dt_conserv + h["dtc"] if gt in _CONSERV else None,
            R=self.diss_A + h["diss_pred"].view(T, n, n) if gt in _PSD else None,
            diag_pre=self.diss_diag + h["diss_pred"] if gt in _DIAG else None,
            scores=self.laplacian_A + h["laplacian_pred"].view(T, n, n) if gt in _LAPLACIAN else None,
            logit_diss=self.log_dt_diss + h["dtd"] if dissipative else None,
            dt_range_conserv=(self.dt_min_cons, self.dt_max_cons), dt_range_diss=(self.dt_min_diss, self.dt_max_diss),
            vec_dt=self.vec_dt)
        if self.projection == "mean":
            v = self.projection_dir.unsqueeze(0)
        elif self.projection == "v":
            v = F.normalize(h["v"], dim=-1)
        else:
            v = None
        out = hc_mix_write(Phi, xs, write, f, v)
        return out.reshape(*lead, n * blk)
