"""Hot-path operators with the reference's import path and names
(hyperconnections/ops/__init__.py:1-4), plus the fused step, the read / mix-write
pair for m backbone blocks, the Pade matrix exponential, MHC's
Sinkhorn-Knopp projection, CGHC's generator assembly and its transition
(generator fused with the exponential)."""

from .expm import expm_t18, matrix_exp
from .fused import stream_mix_fused
from .generator import cghc_generator, cghc_transition
from .rw import hc_mix_write, hc_read
from .sinkhorn import sinkhorn_knopp
from .stream_mix import HAS_TRITON, stream_mix_add

HAS_KERNELS = HAS_TRITON

__all__ = ["HAS_TRITON", "HAS_KERNELS", "stream_mix_add", "expm_t18", "matrix_exp", "stream_mix_fused", "hc_read", "hc_mix_write",
           "sinkhorn_knopp", "cghc_generator", "cghc_transition"]
