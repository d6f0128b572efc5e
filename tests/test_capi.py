"""CPU tests of the C ABI: libhcops.so loads, exports every function that
include/hcops.h declares, and rejects bad arguments on the host before any
launch (no GPU needed for these paths)."""

import ctypes
import os
import re

import pytest

from hyperconnections_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hcops.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hc_[a-z0-9_]+)\s*\(", text)))


def test_library_loads():
    assert _lib.available(), "libhcops.so missing: build it with make -C hyperconnections_b200/csrc"
    assert _lib.lib().hc_abi_version() == _lib.EXPECTED_ABI_VERSION


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/hcops.h but not exported"


def test_binding_covers_header():
    assert set(declared_functions()) == set(_lib._SIGNATURES)


def test_error_strings():
    lib = _lib.lib()
    for code in range(0, 8):
        assert lib.hc_error_string(code)
    assert b"unknown" in lib.hc_error_string(99)


HC_OK, HC_ERR_NULL, HC_ERR_SIZE, HC_ERR_N, HC_ERR_DTYPE, HC_ERR_ALIGN, HC_ERR_SCRATCH = range(7)
FAKE = 0x1000  # never dereferenced: every call below fails host-side checks


@pytest.mark.parametrize(
    "args,want",
    [
        ((FAKE, FAKE, FAKE, None, FAKE, 4, 33, 64, 2, 2, None), HC_ERR_N),  # n <= 32
        ((FAKE, FAKE, FAKE, None, FAKE, 4, 0, 64, 2, 2, None), HC_ERR_N),
        ((FAKE, FAKE, FAKE, None, FAKE, -1, 4, 64, 2, 2, None), HC_ERR_SIZE),
        ((FAKE, FAKE, FAKE, None, FAKE, 4, 4, -5, 2, 2, None), HC_ERR_SIZE),
        ((FAKE, FAKE, FAKE, None, FAKE, 4, 4, 64, 7, 2, None), HC_ERR_DTYPE),
        ((FAKE, FAKE, FAKE, None, FAKE, 4, 4, 64, 2, 1, None), HC_ERR_DTYPE),  # fp16 params, bf16 streams
        ((None, FAKE, FAKE, None, FAKE, 4, 4, 64, 2, 2, None), HC_ERR_NULL),
        ((FAKE + 2, FAKE, FAKE, None, FAKE, 4, 4, 64, 2, 0, None), HC_ERR_ALIGN),
        ((None, None, None, None, None, 0, 4, 64, 2, 2, None), HC_OK),  # empty batch: no work
    ],
)
def test_stream_mix_fwd_argument_checks(args, want):
    assert _lib.lib().hc_stream_mix_fwd(*args) == want


def test_fused_and_expm_argument_checks():
    lib = _lib.lib()
    assert lib.hc_fused_fwd(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 4, 9, 64, 2, None) == HC_ERR_N
    assert lib.hc_fused_fwd(FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, 4, 4, 64, 2, None) == HC_ERR_NULL
    assert lib.hc_fused_bwd(*([FAKE] * 12), 4, 4, 64, 5, None) == HC_ERR_DTYPE
    assert lib.hc_expm_pade_fwd(FAKE, FAKE, 10, 9, None) == HC_ERR_N
    assert lib.hc_expm_pade_fwd(FAKE, FAKE, -1, 4, None) == HC_ERR_SIZE
    assert lib.hc_expm_t18_fwd(FAKE, FAKE, 10, 4, None, 0, 0, None) == HC_ERR_SCRATCH
    words = lib.hc_expm_t18_scratch_words(65536, 4)
    assert 1 <= words <= 1024
    assert lib.hc_expm_t18_fwd(FAKE, FAKE, 65536, 4, FAKE, words - 1, 0, None) == HC_ERR_SCRATCH
    assert lib.hc_expm_t18_scratch_words(10, 9) == 0
    # scaling modes: fwd takes 0 / 1, bwd 0 / 1 / 2 (2 = reuse the forward's partial maxima)
    assert lib.hc_expm_t18_fwd(FAKE, FAKE, 10, 4, FAKE, 1024, 2, None) == HC_ERR_SIZE
    assert lib.hc_expm_t18_bwd(FAKE, FAKE, FAKE, 10, 4, FAKE, 1024, 3, None) == HC_ERR_SIZE
    assert lib.hc_expm_t18_bwd(FAKE, FAKE, FAKE, 10, 4, None, 0, 2, None) == HC_ERR_SCRATCH


def test_read_write_and_sinkhorn_argument_checks():
    lib = _lib.lib()
    assert lib.hc_read_fwd(FAKE, FAKE, FAKE, 4, 4, 5, 64, 2, None) == HC_ERR_N  # m > 4
    assert lib.hc_read_fwd(FAKE, FAKE, FAKE, 4, 9, 1, 64, 2, None) == HC_ERR_N  # n > 8
    assert lib.hc_read_fwd(None, FAKE, FAKE, 4, 4, 1, 64, 2, None) == HC_ERR_NULL
    assert lib.hc_read_fwd(FAKE + 2, FAKE, FAKE, 4, 4, 1, 64, 2, None) == HC_ERR_ALIGN
    assert lib.hc_read_bwd(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 4, 1, 64, 7, None) == HC_ERR_DTYPE
    assert lib.hc_mix_write_fwd(FAKE, FAKE, None, FAKE, None, FAKE, 4, 4, 2, 64, 2, None) == HC_ERR_NULL
    assert lib.hc_mix_write_bwd(*([FAKE] * 11), -1, 4, 2, 64, 2, None) == HC_ERR_SIZE
    assert lib.hc_mix_write_fwd(*([None] * 6), 0, 4, 2, 64, 2, None) == HC_OK  # empty: no work
    assert lib.hc_sinkhorn_fwd(FAKE, FAKE, 10, 9, 20, None) == HC_ERR_N
    assert lib.hc_sinkhorn_fwd(FAKE, FAKE, 10, 4, 257, None) == HC_ERR_SIZE
    assert lib.hc_sinkhorn_bwd(FAKE, None, FAKE, 10, 4, 20, None) == HC_ERR_NULL
    assert lib.hc_sinkhorn_fwd(None, None, 0, 4, 20, None) == HC_OK


def test_cpu_tensors_raise_without_fallback():
    import torch

    from hyperconnections_b200.ops import expm_t18, matrix_exp, stream_mix_add, stream_mix_fused

    with pytest.raises(RuntimeError, match="CUDA"):
        stream_mix_add(torch.randn(2, 4, 4), torch.randn(2, 4, 64), torch.randn(2, 4, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        expm_t18(torch.randn(2, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        matrix_exp(torch.randn(2, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        stream_mix_fused(torch.randn(2, 4, 8), torch.randn(2, 8), torch.randn(2, 4, 4), torch.randn(2, 4),
                         torch.randn(2, 4))
