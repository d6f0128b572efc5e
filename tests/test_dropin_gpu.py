"""Drop-in: the reference's own callers of ``hyperconnections.ops`` run
unchanged on this package's kernels.

With ``hyperconnections.ops`` aliased to ``hyperconnections_b200.ops``
(tests/reference_alias.py; the reference is the unmodified copy installed in
baseline/_ref by baseline/install_reference.py):

* the reference's unit tests of the op, tests/test_ops.py (imports at :17),
  all pass, including the CPU-raises case matched on "CUDA" (:213-218);
* the reference's benchmark, benchmarks/stream_mix_bench.py (imports at :35),
  passes its correctness mode (tolerances :279-280) over its documented
  defaults, N = 4, 8, 16 (16 runs the shared-memory kernels);
* a ContinuousGenHyperConnections layer (cghc.py:394-457) on its
  use_triton=True path, which calls stream_mix_add at cghc.py:363, gives the
  output and every parameter gradient of the same layer on its eager path.

The first two run in subprocesses so that the alias stays out of this process.
"""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from baseline import reference_env  # noqa: E402


@pytest.fixture(autouse=True)
def _needs():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    if not reference_env.available():
        pytest.skip("reference not installed in baseline/_ref (baseline/install_reference.py)")


def _run(args, timeout=900):
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    proc = subprocess.run([sys.executable] + args, cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)
    return proc.returncode, proc.stdout + proc.stderr


ALIAS_LINE = "hyperconnections.ops.stream_mix_add -> hyperconnections_b200.ops.stream_mix"


def test_reference_unit_tests_pass():
    rc, out = _run(["-m", "pytest", "-q", "-p", "tests.reference_alias", "-p", "no:cacheprovider",
                    reference_env.caller_path("tests/test_ops.py")])
    assert ALIAS_LINE in out, out[-2000:]
    assert rc == 0, out[-4000:]
    assert "36 passed" in out, out[-2000:]


def test_reference_benchmark_correctness_mode():
    bench = reference_env.caller_path("benchmarks/stream_mix_bench.py")
    code = ("import runpy, sys; import tests.reference_alias; "
            f"sys.argv = [{bench!r}, '--mode', 'correctness', '--n', '4', '8', '16', '--m', '1', '4', "
            "'--b', '64', '512', '2048', '--embed_dim', '128', '256', '512', '--dtype', 'fp32', 'fp16']; "
            f"runpy.run_path({bench!r}, run_name='__main__')")
    rc, out = _run(["-c", code])
    assert ALIAS_LINE in out, out[-2000:]
    assert rc == 0, out[-4000:]
    assert "All correctness checks passed." in out
    assert "FAIL" not in out


@pytest.mark.parametrize("gen,proj,n,m", [("conservative_psd_diss", "none", 4, 1), ("conservative_diag_diss", "mean", 4, 2),
                                          ("conservative_laplacian", "v", 6, 3), ("laplacian", "mean", 8, 2)])
def test_reference_layer_triton_path_runs_on_b200_ops(gen, proj, n, m):
    """cghc.py:120-124 picks _stream_mix_triton when use_triton and HAS_TRITON:
    with the alias that is this package's stream_mix_add."""
    import hyperconnections_b200.ops as b200_ops

    hc = reference_env.import_reference(ops=b200_ops)
    try:
        CGHC = hc.cghc.ContinuousGenHyperConnections
        E = 64 * m
        torch.manual_seed(11)
        fast = CGHC(n, m, n * E // m, E, torch.nn.Linear(E, E), dt=0.3, generator_type=gen, projection=proj,
                    use_triton=True).cuda()
        eager = CGHC(n, m, n * E // m, E, torch.nn.Linear(E, E), dt=0.3, generator_type=gen, projection=proj,
                     use_triton=False).cuda()
        with torch.no_grad():
            for p in fast.parameters():
                p.add_(0.3 * torch.randn_like(p))
        eager.load_state_dict(fast.state_dict())
        assert fast._stream_mix.__func__ is CGHC._stream_mix_triton
        assert eager._stream_mix.__func__ is CGHC._stream_mix_eager
        x = torch.randn(3, 7, n * E // m, device="cuda")
        g = torch.randn_like(x)
        outs = []
        for layer in (fast, eager):
            xi = x.clone().requires_grad_(True)
            out = layer(xi)
            out.backward(g)
            outs.append((out.detach(), xi.grad, {k: p.grad for k, p in layer.named_parameters() if p.grad is not None}))
        (o1, gx1, p1), (o2, gx2, p2) = outs
        scale = lambda t: max(1.0, t.abs().max().item())  # noqa: E731
        assert (o1 - o2).abs().max().item() <= 1e-5 * scale(o2)
        assert (gx1 - gx2).abs().max().item() <= 1e-5 * scale(gx2)
        assert p1.keys() == p2.keys() and len(p1) > 0
        for k in p1:
            assert (p1[k] - p2[k]).abs().max().item() <= 1e-5 * scale(p2[k]), k
    finally:
        reference_env._forget_reference()
