"""GHC layer on the B200 kernels: drop-in for the reference's
``hyperconnections.ghc.GeneralizedHyperConnections`` (ghc.py:14-128).

Same constructor arguments, parameters and ``state_dict`` keys as the
reference, and the same forward (ghc.py:109-127): ``x [*, n * block]`` ->
``[*, n * block]``. Per token, with x_norm the RMSNorm of every stream row
(ghc.py:84):

    h        = one GEMM of x_norm against the three tanh heads
    W        = s_W * tanh(h_W / sqrt(block)) + W0            [n, m]   (ghc.py:86-90)
    R        = (s_R * tanh(h_R / sqrt(block)) + R0)^T         [m, n]   (ghc.py:92-96)
    H        = s_H * tanh(h_H / sqrt(block)) + H0             [n, n]   (ghc.py:98-102)
    u        = hc_read(R, x)                                  (ghc.py:116)
    f        = module(u)                                      (ghc.py:119)
    x_new    = hc_mix_write(H, x, W, f)  = H x + W f          (ghc.py:122-126)

The written term W f is never materialised and the three Linear heads are one
GEMM. The per-token matrices are computed in float32 (the kernels take float32
weights).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import hc_mix_write, hc_read


class GeneralizedHyperConnections(nn.Module):
    """Generalised hyper-connection layer (see module doc). Args are the
    reference's (ghc.py:15-24)."""

    def __init__(self, n: int, m: int, input_dim: int, embed_dim: int, module: nn.Module, bias: bool = False,
                 elementwise_affine: bool = False):
        super().__init__()
        if embed_dim % m:
            raise ValueError(f"embed_dim ({embed_dim}) must be divisible by m ({m})")
        if input_dim != n * embed_dim // m or (n * embed_dim) % m:
            raise ValueError(f"input_dim must be (n/m)*embed_dim = {n * embed_dim // m}, got {input_dim}")
        self.n, self.m, self.input_dim, self.embed_dim = n, m, input_dim, embed_dim
        self.block_size = embed_dim // m
        self.scaling_factor = math.sqrt(self.block_size)
        blk = self.block_size
        self.write_out = nn.Parameter(torch.empty(n, m))
        self.dynamic_scaling_write_out = nn.Parameter(torch.ones(n, m))
        self.dynamic_scaling_weight_write_out = nn.Linear(blk, m, bias=bias)
        self.read_in = nn.Parameter(torch.empty(n, m))
        self.dynamic_scaling_read_in = nn.Parameter(torch.ones(n, m))
        self.dynamic_scaling_weight_read_in = nn.Linear(blk, m, bias=bias)
        self.stream_mixing = nn.Parameter(torch.empty(n, n))
        self.dynamic_scaling_stream_mixing = nn.Parameter(torch.ones(n, n))
        self.dynamic_scaling_weight_stream_mixing = nn.Linear(blk, n, bias=bias)
        self.norm = nn.RMSNorm(blk, elementwise_affine=elementwise_affine)
        self.module = module
        self.init_weights()

    @torch.no_grad()
    def init_weights(self):
        """Static connections at init (ghc.py:57-80): stream j writes block
        j mod m, the first m streams read the m blocks, the mix is I, and the
        dynamic heads start at zero."""
        n, m = self.n, self.m
        self.write_out.zero_()
        for j in range(n):
            self.write_out[j, j % m] = 1.0
        self.read_in.zero_()
        self.read_in[:m, :m] = torch.eye(m)
        self.stream_mixing.copy_(torch.eye(n))
        for head in self._heads():
            head.weight.zero_()
            if head.bias is not None:
                head.bias.zero_()

    def _heads(self):
        return [self.dynamic_scaling_weight_write_out, self.dynamic_scaling_weight_read_in,
                self.dynamic_scaling_weight_stream_mixing]

    def forward(self, x: torch.Tensor, **kwargs) -> torch.Tensor:
        n, m, blk = self.n, self.m, self.block_size
        lead = x.shape[:-1]
        xs = x.reshape(-1, n, blk)
        T = xs.shape[0]
        heads = self._heads()
        weight = torch.cat([h.weight for h in heads])
        bias = torch.cat([h.bias if h.bias is not None else h.weight.new_zeros(h.out_features) for h in heads])
        h = F.linear(self.norm(xs), weight, bias).float() / self.scaling_factor  # [T, n, 2m + n]
        h_w, h_r, h_s = h.split([m, m, n], dim=-1)
        write = self.dynamic_scaling_write_out * torch.tanh(h_w) + self.write_out
        read = (self.dynamic_scaling_read_in * torch.tanh(h_r) + self.read_in).transpose(1, 2)
        mix = self.dynamic_scaling_stream_mixing * torch.tanh(h_s) + self.stream_mixing
        u = hc_read(read, xs)
        f = self.module(u.reshape(*lead, self.embed_dim), **kwargs).reshape(T, m, blk)
        return hc_mix_write(mix, xs, write, f).reshape(*lead, n * blk)
