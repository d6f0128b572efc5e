"""A bounded wait that gives up is reported to the caller.

hc_debug_set_wait_limit(1) makes the data waits of the ring kernels and the
grid barrier of the cooperative expm forward give up after one poll (the
ring's exit drain keeps its full limit, so no copy outlives its CTA). The
kernel returns, the give-up lands in the library's status word, every later
entry point call returns HC_ERR_TIMEOUT without launching and the Python ops
raise, until hc_wait_timeouts(reset) clears it; after the reset the same call
reproduces the result of a normal run bit for bit.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from hyperconnections_b200 import _lib

    handle = _lib.lib()
    _lib.wait_timeouts(reset=True)
    yield handle
    assert handle.hc_debug_set_wait_limit(0) == 0
    _lib.wait_timeouts(reset=True)


def _status():
    from hyperconnections_b200 import _lib

    return _lib.timeout_status()


def _force_give_up(lib, launch, tries=5):
    """Launch with a one-poll wait limit until some wait has given up."""
    assert lib.hc_debug_set_wait_limit(1) == 0
    try:
        for _ in range(tries):
            rc = launch()
            torch.cuda.synchronize()
            if rc != 0 or _status() > 0:
                break
    finally:
        assert lib.hc_debug_set_wait_limit(0) == 0
    torch.cuda.synchronize()


def test_ring_give_up_is_sticky_until_reset(lib):
    from hyperconnections_b200 import _lib
    from hyperconnections_b200.ops import stream_mix_fused

    from bench import fused_workload

    T, n, D = 16384, 4, 768
    x, f, H, a, b, _, _ = (t.cuda() for t in fused_workload(T, n, D, seed=5))
    u = torch.empty(T, D, dtype=x.dtype, device="cuda")
    xo = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream

    def launch():
        return lib.hc_fused_fwd(x.data_ptr(), f.data_ptr(), H.data_ptr(), a.data_ptr(), b.data_ptr(), u.data_ptr(),
                                xo.data_ptr(), T, n, D, _lib.HC_DTYPE_BF16, stream)

    assert launch() == 0
    torch.cuda.synchronize()
    assert _status() == 0
    u_ref, xo_ref = u.clone(), xo.clone()

    _force_give_up(lib, launch)
    assert _status() > 0, "no wait gave up with a one-poll limit"
    # later calls report it without launching, whatever the op
    assert launch() == _lib.HC_ERR_TIMEOUT
    assert lib.hc_expm_pade_fwd(H.data_ptr(), H.data_ptr(), 0, 4, stream) == _lib.HC_ERR_TIMEOUT
    with pytest.raises(RuntimeError, match="gave up"):
        stream_mix_fused(x, f, H, a, b)
    count = ctypes.c_uint(0)
    assert lib.hc_wait_timeouts(ctypes.byref(count), 1) == 0
    assert count.value > 0
    assert _status() == 0 and _lib.wait_timeouts() == 0
    # cleared: the full limit again, and the result of a normal run
    assert launch() == 0
    torch.cuda.synchronize()
    assert torch.equal(u, u_ref) and torch.equal(xo, xo_ref)
    assert _lib.wait_timeouts() == 0


def test_expm_grid_barrier_give_up_is_reported(lib):
    from hyperconnections_b200 import _lib
    from hyperconnections_b200.ops import expm_t18

    from bench import expm_workload

    A, _ = expm_workload(65536, 4)
    A = A.cuda()
    E = torch.empty_like(A)
    words = lib.hc_expm_t18_scratch_words(A.shape[0], 4)
    scratch = torch.empty(words, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def launch():
        return lib.hc_expm_t18_fwd(A.data_ptr(), E.data_ptr(), A.shape[0], 4, scratch.data_ptr(), words, 0, stream)

    assert launch() == 0
    torch.cuda.synchronize()
    E_ref = E.clone()
    _force_give_up(lib, launch)
    # the first CTA to arrive cannot see every CTA arrive within one poll
    assert _status() > 0
    with pytest.raises(RuntimeError, match="gave up"):
        expm_t18(A)
    assert _lib.wait_timeouts(reset=True) > 0
    assert launch() == 0
    torch.cuda.synchronize()
    assert torch.equal(E, E_ref)
    assert _lib.wait_timeouts() == 0
