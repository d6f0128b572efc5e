"""The shared-memory ring at the edges of its geometry.

hc_debug_set_mix_tuning overrides the automatic choices: the item target (small
tokens grouped per item, or tokens cut into slices), the number of stages and
the number of consumer warps. Results must not depend on them: at every
setting below the fused step, stream_mix_add and the read / mix-write pair
match the oracle, and no bounded wait gives up (the minimal ring of 3 stages
with 1 consumer, many consumers on few stages, one token per item, many
tokens per item)."""

import numpy as np
import pytest
import torch

from oracle import rw as orw
from oracle import stream_mix as omix
from tests.parity import assert_half

pytestmark = pytest.mark.gpu

SETTINGS = [  # (item target bytes, stages, consumer warps, producer lanes); 0 = automatic
    (0, 3, 1, 0), (0, 3, 0, 0), (0, 4, 2, 0), (0, 0, 1, 0), (0, 0, 15, 0), (2048, 0, 0, 0), (65536, 0, 0, 0),
    (65536, 5, 3, 0), (1, 0, 0, 0), (0, 32, 0, 0), (0, 0, 0, 2), (0, 0, 0, 4), (16384, 0, 0, 4), (0, 3, 1, 3),
]


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


@pytest.fixture
def lib():
    from hyperconnections_b200 import _lib

    handle = _lib.lib()
    yield handle
    assert handle.hc_debug_set_mix_tuning(0, 0, 0, 0) == 0


def np64(t):
    return t.detach().double().cpu().numpy()


def half_close(got, ref, what):
    assert_half(got, ref, what)


def rel_close(got, ref, what):
    err = np.abs(np64(got) - ref).max()
    assert err <= 1e-5 * max(1.0, np.abs(ref).max()), f"{what}: {err:.3e}"


@pytest.mark.parametrize("setting", SETTINGS, ids=[f"t{a}-s{b}-w{c}-p{d}" for a, b, c, d in SETTINGS])
@pytest.mark.parametrize("D", [64, 768, 4096])
def test_results_do_not_depend_on_geometry(lib, setting, D):
    from hyperconnections_b200 import _lib
    from hyperconnections_b200.ops import hc_mix_write, hc_read, stream_mix_add, stream_mix_fused

    assert lib.hc_debug_set_mix_tuning(*setting) == 0
    g = torch.Generator().manual_seed(D)
    T, n = 700, 4
    x = torch.randn(T, n, D, generator=g).bfloat16()
    f = torch.randn(T, D, generator=g).bfloat16()
    H = torch.randn(T, n, n, generator=g) * 0.5
    a, b = torch.rand(T, n, generator=g), torch.rand(T, n, generator=g)
    gu, gx = torch.randn(T, D, generator=g).bfloat16(), torch.randn(T, n, D, generator=g).bfloat16()
    leaves = [t.cuda().requires_grad_(True) for t in (x, f, H, a, b)]
    u, xo = stream_mix_fused(*leaves)
    torch.autograd.backward([u, xo], [gu.cuda(), gx.cuda()])
    n64 = [np64(t) for t in (x, f, H, a, b, gu, gx)]
    ru, rx = omix.fused_fwd(*n64[:5])
    rg = omix.fused_bwd(n64[5], n64[6], *n64[:5])
    half_close(u, ru, "u")
    half_close(xo, rx, "x_out")
    half_close(leaves[0].grad, rg[0], "grad_x")
    half_close(leaves[1].grad, rg[1], "grad_f")
    for k, name in ((2, "grad_H"), (3, "grad_alpha"), (4, "grad_beta")):
        rel_close(leaves[k].grad, rg[k], name)

    # stream_mix_add with a projection direction, fp32
    v = torch.nn.functional.normalize(torch.randn(T, n, generator=g), dim=-1)
    Y = torch.randn(T, n, D, generator=g)
    ts = [t.cuda().requires_grad_(True) for t in (H, x.float(), Y, v)]
    out = stream_mix_add(*ts)
    out.backward(gx.float().cuda())
    rel_close(out, omix.stream_mix_fwd(np64(H), n64[0], np64(Y), np64(v)), "stream_mix out")
    rP, rxg, _, rv = omix.stream_mix_bwd(n64[6], np64(H), n64[0], np64(v))
    rel_close(ts[0].grad, rP, "stream_mix grad_Phi")
    rel_close(ts[1].grad, rxg, "stream_mix grad_x")
    rel_close(ts[3].grad, rv, "stream_mix grad_v")

    # read / mix-write with m = 2
    m = 2
    R, W = torch.rand(T, m, n, generator=g), torch.rand(T, n, m, generator=g)
    f2 = torch.randn(T, m, D, generator=g).bfloat16()
    ts = [t.cuda().requires_grad_(True) for t in (R, x, W, f2, H)]
    xm = x.cuda().requires_grad_(True)  # its own leaf: each kernel's grad_x is checked before any sum
    ur = hc_read(ts[0], ts[1])
    xw = hc_mix_write(ts[4], xm, ts[2], ts[3])
    g2 = torch.randn(T, m, D, generator=g).bfloat16()
    torch.autograd.backward([ur, xw], [g2.cuda(), gx.cuda()])
    half_close(ur, orw.read_fwd(np64(R), n64[0]), "read u")
    half_close(xw, orw.mix_write_fwd(np64(H), n64[0], np64(W), np64(f2)), "mix-write out")
    rR, rx_r = orw.read_bwd(np64(g2), np64(R), n64[0])
    rH, rx_m, rW, rf, _ = orw.mix_write_bwd(n64[6], np64(H), n64[0], np64(W), np64(f2))
    rel_close(ts[0].grad, rR, "grad_R")
    rel_close(ts[2].grad, rW, "grad_W")
    rel_close(ts[4].grad, rH, "grad_H (mix-write)")
    half_close(ts[1].grad, rx_r, "grad_x (read)")
    half_close(xm.grad, rx_m, "grad_x (mix-write)")
    half_close(ts[3].grad, rf, "grad_f (mix-write)")
    assert _lib.wait_timeouts(reset=True) == 0
