"""The operators run inside CUDA-graph capture: no host synchronisation and no
allocation inside the C calls (outputs and scratch come from torch's caching
allocator). A captured forward + backward replayed on new inputs must give
exactly the results of eager execution of the same calls."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def _graph_vs_eager(make_inputs, step):
    """Capture step(static inputs) once, then for two fresh input sets copy
    them in, replay, and compare every output with an eager call."""
    static = make_inputs(0)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up on a side stream, as torch requires before capture
        for _ in range(2):
            step(*static)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = step(*static)
    for seed in (1, 2):
        fresh = make_inputs(seed)
        for dst, src in zip(static, fresh):
            dst.copy_(src)
        g.replay()
        ref = step(*fresh)
        torch.cuda.synchronize()
        for got, want in zip(outs, ref):
            assert torch.equal(got, want)


def test_fused_step_in_a_graph():
    from hyperconnections_b200.ops import stream_mix_fused

    T, n, D = 2048, 4, 768

    def make(seed):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(T, n, D, generator=g).bfloat16()
        f = torch.randn(T, D, generator=g).bfloat16()
        H = torch.linalg.matrix_exp(torch.randn(T, n, n, generator=g) * 0.3)
        a = torch.softmax(torch.randn(T, n, generator=g), -1)
        b = torch.softmax(torch.randn(T, n, generator=g), -1)
        gu = torch.randn(T, D, generator=g).bfloat16()
        gx = torch.randn(T, n, D, generator=g).bfloat16()
        return [t.cuda() for t in (x, f, H, a, b, gu, gx)]

    def step(x, f, H, a, b, gu, gx):
        leaves = [t.detach().requires_grad_(True) for t in (x, f, H, a, b)]
        u, xo = stream_mix_fused(*leaves)
        grads = torch.autograd.grad([u, xo], leaves, [gu, gx])
        return [u.detach(), xo.detach(), *grads]

    _graph_vs_eager(make, step)


def test_stream_mix_and_expm_in_a_graph():
    from hyperconnections_b200.ops import expm_t18, stream_mix_add

    B, N, D = 1000, 6, 256

    def make(seed):
        g = torch.Generator().manual_seed(seed)
        A = 0.5 * torch.randn(B, N, N, generator=g)
        x, Y, G = (torch.randn(B, N, D, generator=g) for _ in range(3))
        v = torch.nn.functional.normalize(torch.randn(B, N, generator=g), dim=-1)
        GE = torch.randn(B, N, N, generator=g)
        return [t.cuda() for t in (A, x, Y, v, G, GE)]

    def step(A, x, Y, v, G, GE):
        Al = A.detach().requires_grad_(True)
        Phi = expm_t18(Al)
        leaves = [t.detach().requires_grad_(True) for t in (x, Y, v)]
        out = stream_mix_add(Phi, *leaves)
        gPhi, gx, gY, gv = torch.autograd.grad(out, [Phi, *leaves], G, retain_graph=True)
        (gA,) = torch.autograd.grad(Phi, Al, GE)
        return [out.detach(), gPhi, gx, gY, gv, gA]

    _graph_vs_eager(make, step)


def test_read_mix_write_in_a_graph():
    from hyperconnections_b200.ops import hc_mix_write, hc_read

    T, n, m, D = 1500, 4, 2, 512

    def make(seed):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(T, n, D, generator=g).bfloat16()
        f = torch.randn(T, m, D, generator=g).bfloat16()
        R, W = torch.rand(T, m, n, generator=g), torch.rand(T, n, m, generator=g)
        H = torch.randn(T, n, n, generator=g)
        gu, gx = torch.randn(T, m, D, generator=g).bfloat16(), torch.randn(T, n, D, generator=g).bfloat16()
        return [t.cuda() for t in (x, f, R, W, H, gu, gx)]

    def step(x, f, R, W, H, gu, gx):
        leaves = [t.detach().requires_grad_(True) for t in (x, f, R, W, H)]
        u = hc_read(leaves[2], leaves[0])
        xo = hc_mix_write(leaves[4], leaves[0], leaves[3], leaves[1])
        grads = torch.autograd.grad([u, xo], leaves, [gu, gx])
        return [u.detach(), xo.detach(), *grads]

    _graph_vs_eager(make, step)
