"""ctypes binding of libhcops.so, the C ABI declared in include/hcops.h.

This module is the only place that touches the shared library. It resolves
every entry point once, fixes its argument types, and turns non-zero status
codes into RuntimeError. There is deliberately no fallback: when the library
is missing or a tensor is not on a CUDA device, the callers in
``hyperconnections_b200.ops`` raise instead of computing anything elsewhere.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

# The in-tree build, unless HC_LIBHCOPS names another build of the same ABI
# (read once, when this module is imported: importing the package loads the
# library, so a later change of LIB_PATH does not switch builds).
LIB_PATH = os.environ.get("HC_LIBHCOPS") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhcops.so")

HC_DTYPE_F32 = 0
HC_DTYPE_F16 = 1
HC_DTYPE_BF16 = 2

_DTYPE_CODE = {
    torch.float32: HC_DTYPE_F32,
    torch.float16: HC_DTYPE_F16,
    torch.bfloat16: HC_DTYPE_BF16,
}

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/hcops.h
_SIGNATURES = {
    "hc_error_string": (ctypes.c_char_p, [_c_int]),
    "hc_abi_version": (_c_int, []),
    "hc_wait_timeouts": (_c_int, [ctypes.POINTER(ctypes.c_uint), _c_int]),
    "hc_timeout_status": (_c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "hc_debug_set_mix_tuning": (_c_int, [_c_int, _c_int, _c_int, _c_int]),
    "hc_debug_set_wait_limit": (_c_int, [ctypes.c_uint]),
    "hc_debug_ring_geometry": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64, _c_int, ctypes.POINTER(_c_int), _c_int],
    ),
    "hc_expm_t18_scratch_words": (_c_i64, [_c_i64, _c_int]),
    "hc_expm_t18_fwd": (_c_int, [_vp, _vp, _c_i64, _c_int, _vp, _c_i64, _c_int, _vp]),
    "hc_expm_t18_fwd_noalloc": (_c_int, [_vp, _vp, _c_i64, _c_int, _vp]),
    "hc_expm_t18_bwd": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _vp, _c_i64, _c_int, _vp]),
    "hc_expm_pade_fwd": (_c_int, [_vp, _vp, _c_i64, _c_int, _vp]),
    "hc_expm_pade_bwd": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _vp]),
    "hc_stream_mix_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_int, _c_i64, _c_int, _c_int, _vp]),
    "hc_stream_mix_bwd": (
        _c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_int, _c_i64, _c_int, _c_int, _vp],
    ),
    "hc_fused_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_int, _c_i64, _c_int, _vp]),
    "hc_fused_bwd": (
        _c_int,
        [_vp] * 12 + [_c_i64, _c_int, _c_i64, _c_int, _vp],
    ),
    "hc_sinkhorn_fwd": (_c_int, [_vp, _vp, _c_i64, _c_int, _c_int, _vp]),
    "hc_sinkhorn_bwd": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _c_int, _vp]),
    "hc_cghc_generator_fwd": (_c_int, [_vp] * 7 + [_c_i64, _c_int, _c_int, _c_int] + [ctypes.c_float] * 4 + [_vp]),
    "hc_cghc_generator_bwd": (_c_int, [_vp] * 13 + [_c_i64, _c_int, _c_int, _c_int] + [ctypes.c_float] * 4 + [_vp]),
    "hc_cghc_transition_fwd": (_c_int, [_vp] * 7 + [_c_i64, _c_int, _c_int, _c_int] + [ctypes.c_float] * 4 + [_vp]),
    "hc_cghc_transition_bwd": (_c_int, [_vp] * 13 + [_c_i64, _c_int, _c_int, _c_int] + [ctypes.c_float] * 4 + [_vp]),
    "hc_read_fwd": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _c_int, _c_i64, _c_int, _vp]),
    "hc_read_bwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_i64, _c_int, _c_int, _c_i64, _c_int, _vp]),
    "hc_mix_write_fwd": (_c_int, [_vp] * 6 + [_c_i64, _c_int, _c_int, _c_i64, _c_int, _vp]),
    "hc_mix_write_bwd": (_c_int, [_vp] * 11 + [_c_i64, _c_int, _c_int, _c_i64, _c_int, _vp]),
}

EXPECTED_ABI_VERSION = 7

_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def _load() -> Optional[ctypes.CDLL]:
    global _lib, _load_error
    if _lib is not None or _load_error is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        _load_error = f"{LIB_PATH} is not built (run `make -C hyperconnections_b200/csrc`)"
        return None
    try:
        lib = ctypes.CDLL(LIB_PATH)
    except OSError as exc:  # pragma: no cover - depends on the environment
        _load_error = f"cannot load {LIB_PATH}: {exc}"
        return None
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.hc_abi_version() != EXPECTED_ABI_VERSION:
        _load_error = "libhcops.so ABI version mismatch; rebuild it"
        return None
    _lib = lib
    return _lib


_ext = None


def torch_ext():
    """The C++ autograd ops over this library (_hcops_torch.so, built beside
    it by the same Makefile); raises RuntimeError when it is missing."""
    global _ext
    if _ext is None:
        lib()  # the extension links libhcops.so: load (and version-check) it first
        try:
            from . import _hcops_torch as ext
        except ImportError as exc:
            raise RuntimeError(f"hyperconnections_b200 torch ops unavailable: {exc} "
                               "(run `make -C hyperconnections_b200/csrc`)") from None
        if ext.abi_version() != EXPECTED_ABI_VERSION:
            raise RuntimeError("_hcops_torch.so was built against another libhcops.so ABI; rebuild it")
        _ext = ext
    return _ext


def available() -> bool:
    """True when libhcops.so is present and loadable."""
    return _load() is not None


def lib() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError when it is unavailable."""
    handle = _load()
    if handle is None:
        raise RuntimeError(f"hyperconnections_b200 CUDA kernels unavailable: {_load_error}")
    return handle


def check(rc: int, what: str) -> None:
    """Raise RuntimeError for a non-zero hcops status code."""
    if rc != 0:
        msg = lib().hc_error_string(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (hcops status {rc})")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    """Device address of a tensor (None stays None -> NULL)."""
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """Raw cudaStream_t of torch's current stream on the tensor's device."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


class on_device:
    """Make the tensor's device current for a launch; a no-op (no device
    switch) when it already is, the common case."""

    __slots__ = ("idx", "prev")

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


HC_ERR_TIMEOUT = 8


def wait_timeouts(reset: bool = False) -> int:
    """Number of bounded kernel waits that gave up on the current device
    (synchronises the device). reset=True also clears the sticky status that
    makes every entry point return HC_ERR_TIMEOUT after a give-up."""
    count = ctypes.c_uint(0)
    check(lib().hc_wait_timeouts(ctypes.byref(count), 1 if reset else 0), "hc_wait_timeouts")
    return int(count.value)


def timeout_status() -> int:
    """Give-ups recorded so far by kernels that have reached them (no
    synchronisation)."""
    count = ctypes.c_uint(0)
    check(lib().hc_timeout_status(ctypes.byref(count)), "hc_timeout_status")
    return int(count.value)


def raise_if_timed_out(what: str) -> None:
    """RuntimeError when a kernel has already recorded a give-up (checked at
    the end of a backward pass by the autograd wrappers; no synchronisation)."""
    if timeout_status():
        check(HC_ERR_TIMEOUT, what)
