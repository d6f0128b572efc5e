"""GPU parity of CGHC's fused transition (hc_cghc_transition_fwd/bwd via
ops.cghc_transition): generator assembly and Pade [7/7] exponential in one
kernel per direction. It runs the same device code on the same values as the
two launches cghc_generator -> matrix_exp, so Phi and every gradient must be
bit for bit theirs (both are pinned to the reference separately:
tests/test_generator_gpu.py, tests/test_expm_gpu.py). It is also checked
against the float64 oracle of the generator composed with a float64 matrix
exponential, and through the CGHC layer against the reference layer's fixtures
(tests/test_cghc_module.py)."""

import itertools

import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = {"M": "M", "lc": "logit_conserv", "R": "R", "dpre": "diag_pre", "S": "scores", "ld": "logit_diss"}
TERMS = [c for r in range(1, 5) for c in itertools.combinations(("M", "R", "dpre", "S"), r)]


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def inputs(n, T, terms, vec, seed):
    g = torch.Generator().manual_seed(seed)
    nd = n if vec else 1
    ins = {}
    for k in terms:
        shape = (T, n) if k == "dpre" else (T, n, n)
        ins[k] = 0.7 * torch.randn(*shape, generator=g)
    if "M" in terms:
        ins["lc"] = torch.randn(T, nd, generator=g)
    if set(terms) & {"R", "dpre", "S"}:
        ins["ld"] = torch.randn(T, nd, generator=g)
    return ins, torch.randn(T, n, n, generator=g)


def run(fn, ins, G, vec, ranges):
    leaves = {k: v.cuda().requires_grad_(True) for k, v in ins.items()}
    out = fn(**{NAMES[k]: v for k, v in leaves.items()}, dt_range_conserv=ranges[:2], dt_range_diss=ranges[2:],
             vec_dt=vec)
    out.backward(G.cuda())
    return out.detach(), {k: v.grad for k, v in leaves.items()}


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("vec", [False, True])
@pytest.mark.parametrize("terms", TERMS, ids=["+".join(t) for t in TERMS])
def test_bitwise_equal_to_two_launches(n, vec, terms):
    from hyperconnections_b200.ops import cghc_generator, cghc_transition, matrix_exp

    ranges = (0.001, 1.0, 0.01, 0.5)
    T = 517  # not a multiple of the tokens per CTA
    ins, G = inputs(n, T, terms, vec, seed=100 * n + len(terms) + int(vec))
    Phi_f, grads_f = run(cghc_transition, ins, G, vec, ranges)
    Phi_u, grads_u = run(lambda **kw: matrix_exp(cghc_generator(**kw)), ins, G, vec, ranges)
    assert torch.equal(Phi_f, Phi_u)
    assert grads_f.keys() == grads_u.keys()
    for k in grads_f:
        assert torch.equal(grads_f[k], grads_u[k]), k


def test_against_float64_oracle():
    """Phi and every gradient against the float64 generator oracle composed
    with torch.linalg.matrix_exp in float64 (the exponential to double
    precision; the Pade [7/7] approximant is within 1e-5 of it), gradients by
    autograd through both."""
    from hyperconnections_b200.ops import cghc_transition
    from oracle import generator as ogen

    n, T, vec = 4, 64, True
    ranges = (0.001, 1.0, 0.001, 1.0)
    ins, G = inputs(n, T, ("M", "R", "S"), vec, seed=7)
    Phi, grads = run(cghc_transition, ins, G, vec, ranges)
    leaves = {k: v.double().requires_grad_(True) for k, v in ins.items()}
    ref = torch.linalg.matrix_exp(ogen.generator(**leaves, ranges=ranges, vec_dt=vec))
    ref.backward(G.double())
    got = Phi.double().cpu()
    rel = torch.linalg.matrix_norm(got - ref.detach()) / torch.linalg.matrix_norm(ref.detach())
    assert rel.max().item() <= 1e-5
    for k, v in leaves.items():
        err = (grads[k].double().cpu() - v.grad).abs().max().item()
        assert err <= 1e-5 * max(1.0, v.grad.abs().max().item()), k


def test_argument_errors():
    from hyperconnections_b200 import _lib

    lib = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    Phi = torch.empty(4, 4, 4, device="cuda")
    M = torch.randn(4, 4, 4, device="cuda")
    lc = torch.randn(4, 1, device="cuda")
    # conservative without its dt logit
    assert lib.hc_cghc_transition_fwd(M.data_ptr(), None, None, None, None, None, Phi.data_ptr(), 4, 4, 0, 1,
                                      0.001, 1.0, 0.001, 1.0, st) == 1
    assert lib.hc_cghc_transition_fwd(M.data_ptr(), lc.data_ptr(), None, None, None, None, Phi.data_ptr(), 4, 9, 0,
                                      1, 0.001, 1.0, 0.001, 1.0, st) == 3
    assert lib.hc_cghc_transition_fwd(M.data_ptr(), lc.data_ptr(), None, None, None, None, None, 4, 4, 0, 1,
                                      0.001, 1.0, 0.001, 1.0, st) == 1
    assert lib.hc_cghc_transition_fwd(M.data_ptr(), lc.data_ptr(), None, None, None, None, Phi.data_ptr(), 0, 4, 0,
                                      1, 0.001, 1.0, 0.001, 1.0, st) == 0
