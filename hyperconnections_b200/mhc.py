"""MHC layer on the B200 kernels: drop-in for the reference's
``hyperconnections.mhc.ManifoldHyperConnections`` (mhc.py:21-150).

Same constructor arguments, parameters and ``state_dict`` keys as the
reference, and the same forward (mhc.py:127-149): ``x [*, n * block]`` ->
``[*, n * block]``. Per token, with x_norm the RMSNorm of the flattened
streams (mhc.py:106):

    h     = one GEMM of x_norm against the read, write and mixing heads
    R     = sigmoid(a_R h_R + R0)^T                [m, n]   (mhc.py:113-118)
    W     = 2 sigmoid(a_W h_W + W0)                [n, m]   (mhc.py:114-119)
    H     = sinkhorn_knopp(a_H h_H + H0, iters)    [n, n]   (mhc.py:115-120, :97-102)
    u     = hc_read(R, x)                          (mhc.py:138)
    f     = module(u)                              (mhc.py:141)
    x_new = hc_mix_write(H, x, W, f) = H x + W f   (mhc.py:144-149)

The doubly stochastic projection is one kernel pair instead of 2 x iters
elementwise passes, the written term W f is never materialised and the three
heads are one GEMM. Deliberate difference: the per-token matrices stay float32
(the reference casts them to the stream dtype, mhc.py:130-132).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import hc_mix_write, hc_read, sinkhorn_knopp


class ManifoldHyperConnections(nn.Module):
    """Manifold-constrained hyper-connection layer (see module doc). Args are
    the reference's (mhc.py:22-33)."""

    def __init__(self, n: int, m: int, input_dim: int, embed_dim: int, module: nn.Module, bias: bool = False,
                 elementwise_affine: bool = False, sinkhorn_iters: int = 20, sinkhorn_bias_init: float = 0.0):
        super().__init__()
        if embed_dim % m:
            raise ValueError(f"embed_dim ({embed_dim}) must be divisible by m ({m})")
        if input_dim != n * embed_dim // m or (n * embed_dim) % m:
            raise ValueError(f"input_dim must be (n/m)*embed_dim = {n * embed_dim // m}, got {input_dim}")
        self.n, self.m, self.input_dim, self.embed_dim = n, m, input_dim, embed_dim
        self.sinkhorn_iters, self.sinkhorn_bias_init = sinkhorn_iters, sinkhorn_bias_init
        self.block_size = embed_dim // m
        self.read_in = nn.Parameter(torch.empty(n, m))
        self.alpha_read_in = nn.Parameter(torch.empty(1))
        self.write_out = nn.Parameter(torch.empty(n, m))
        self.alpha_write_out = nn.Parameter(torch.empty(1))
        self.stream_mixing = nn.Parameter(torch.empty(n, n))
        self.alpha_stream_mixing = nn.Parameter(torch.empty(1))
        self.proj_read_in = nn.Linear(input_dim, n * m, bias=bias)
        self.proj_write_out = nn.Linear(input_dim, n * m, bias=bias)
        self.proj_stream_mixing = nn.Linear(input_dim, n * n, bias=bias)
        self.norm = nn.RMSNorm(input_dim, elementwise_affine=elementwise_affine)
        self.module = module
        self.init_weights()

    @torch.no_grad()
    def init_weights(self):
        """The reference's initial state (mhc.py:68-95): read weights at
        sigmoid^-1(1/n), write weights at 2 sigmoid(0) = 1, mixing logits at
        sinkhorn_bias_init * I, gates 0.01, heads with std-0.01 weights."""
        n = self.n
        self.read_in.fill_(math.log(1.0 / (n - 1)) if n > 1 else 10.0)
        self.write_out.zero_()
        self.stream_mixing.copy_(self.sinkhorn_bias_init * torch.eye(n))
        for alpha in (self.alpha_read_in, self.alpha_write_out, self.alpha_stream_mixing):
            alpha.fill_(0.01)
        for head in self._heads():
            nn.init.trunc_normal_(head.weight, std=0.01)
            if head.bias is not None:
                head.bias.zero_()

    def _heads(self):
        return [self.proj_read_in, self.proj_write_out, self.proj_stream_mixing]

    def forward(self, x: torch.Tensor, **kwargs) -> torch.Tensor:
        n, m, blk = self.n, self.m, self.block_size
        lead = x.shape[:-1]
        xs = x.reshape(-1, n, blk)
        T = xs.shape[0]
        heads = self._heads()
        weight = torch.cat([h.weight for h in heads])
        bias = torch.cat([h.bias if h.bias is not None else h.weight.new_zeros(h.out_features) for h in heads])
        h = F.linear(self.norm(xs.reshape(T, n * blk)), weight, bias).float()
        h_r, h_w, h_s = h.split([n * m, n * m, n * n], dim=-1)
        read = torch.sigmoid(self.alpha_read_in * h_r.view(T, n, m) + self.read_in).transpose(1, 2)
        write = 2.0 * torch.sigmoid(self.alpha_write_out * h_w.view(T, n, m) + self.write_out)
        mix = sinkhorn_knopp(self.alpha_stream_mixing * h_s.view(T, n, n) + self.stream_mixing, self.sinkhorn_iters)
        u = hc_read(read, xs)
        f = self.module(u.reshape(*lead, self.embed_dim), **kwargs).reshape(T, m, blk)
        return hc_mix_write(mix, xs, write, f).reshape(*lead, n * blk)
