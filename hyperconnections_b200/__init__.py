"""B200 (sm_100a) kernels for the hyper-connections hot path: batched
small-matrix exponential and fused stream mixing, behind the reference's
``hyperconnections.ops`` interface."""

from . import ops
from .ops import HAS_TRITON, expm_t18, matrix_exp, stream_mix_add, stream_mix_fused

__all__ = ["ops", "HAS_TRITON", "expm_t18", "matrix_exp", "stream_mix_add", "stream_mix_fused"]
