"""GPU test of hc_expm_t18_fwd_noalloc, the entry point for callers that
cannot allocate device memory (a plugin or FFI caller that only gets pointers
from a host framework owning all device memory, or a loop that must not call
cudaMalloc because it can synchronise the device).

It is called through the C ABI (ctypes) with caller-owned inputs and outputs
only, and its result is compared with hc_expm_t18_fwd (the same computation
with caller scratch) on two calls in a row. The first call uses large norms
(scaling exponent > 0) and the second small ones, so partial maxima left in
the library's shared array by the first call would change the second result
if they leaked into it. This file is named to be collected last.
"""

import numpy as np
import pytest
import torch

from oracle import expm as oexpm

pytestmark = pytest.mark.gpu

TOL = 1e-5  # relative Frobenius error per matrix, as in the other expm tests


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def _with_scratch(lib, A, E):
    batch, n, _ = A.shape
    words = lib.hc_expm_t18_scratch_words(batch, n)
    scratch = torch.empty(words, dtype=torch.float32, device=A.device)
    rc = lib.hc_expm_t18_fwd(A.data_ptr(), E.data_ptr(), batch, n, scratch.data_ptr(), words, 0,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hc_error_string(rc)


def _no_alloc(lib, A, E):
    batch, n, _ = A.shape
    rc = lib.hc_expm_t18_fwd_noalloc(A.data_ptr(), E.data_ptr(), batch, n,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hc_error_string(rc)


def test_no_alloc_matches_scratch_entry_point_on_two_calls():
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(5)
    first = (torch.randn(70000, 4, 4, generator=g) * 3.0).to(dev)   # ||A||_1 up to ~30: s > 0
    second = (0.1 * torch.randn(1000, 3, 3, generator=g)).to(dev)   # small norms: s = 0
    for A in (first, second):
        E_ref = torch.empty_like(A)
        E_new = torch.full_like(A, float("nan"))
        _with_scratch(lib, A, E_ref)
        _no_alloc(lib, A, E_new)
        torch.cuda.synchronize()
        got, ref = E_new.cpu().numpy(), E_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert oexpm.rel_fro(got, ref) < TOL
        assert oexpm.rel_fro(got, oexpm.expm_t18(A.cpu().numpy())) < TOL
    assert _lib.wait_timeouts() == 0


def test_no_alloc_rejects_bad_arguments():
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    A = torch.zeros(4, 9, 9, device="cuda:0")
    assert lib.hc_expm_t18_fwd_noalloc(A.data_ptr(), A.data_ptr(), 4, 9, None) == 3  # HC_ERR_UNSUPPORTED_N
    too_many = (1 << 34) + 1
    assert lib.hc_expm_t18_fwd_noalloc(A.data_ptr(), A.data_ptr(), too_many, 4, None) == 2  # HC_ERR_BAD_SIZE
