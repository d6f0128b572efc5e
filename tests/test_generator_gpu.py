"""GPU parity of CGHC's generator assembly (hc_cghc_generator_fwd/bwd via
ops.cghc_generator) against the reference layer's own compute_generator
(hyperconnections/cghc.py:219-315; fixtures tests/golden/generator.npz) and
the float64 oracle (oracle.generator). Float32: A and every gradient to 1e-5
relative to the largest magnitude."""

import itertools

import numpy as np
import pytest
import torch

from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

GEN = load_golden("generator.npz")
CASES = sorted({k.split("_")[0] for k in GEN})
KW = {"M": "M", "lc": "logit_conserv", "R": "R", "dpre": "diag_pre", "S": "scores", "ld": "logit_diss"}


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


def close(got, ref, what):
    got = got.detach().double().cpu().numpy()
    err = np.abs(got - ref).max()
    bound = 1e-5 * max(1.0, np.abs(ref).max())
    assert err <= bound, f"{what}: max err {err:.3e} > {bound:.3e}"


def run(ins, ranges, vec, G):
    from hyperconnections_b200.ops import cghc_generator

    leaves = {k: v.cuda().requires_grad_(True) for k, v in ins.items()}
    A = cghc_generator(**{KW[k]: v for k, v in leaves.items()}, dt_range_conserv=ranges[:2],
                       dt_range_diss=ranges[2:], vec_dt=vec)
    A.backward(G.cuda())
    return A, {k: v.grad for k, v in leaves.items()}


@pytest.mark.parametrize("case", CASES)
def test_matches_reference_layer(case):
    g = lambda name: GEN[f"{case}_{name}"]  # noqa: E731
    ins = {k: torch.from_numpy(g(k)) for k in KW if f"{case}_{k}" in GEN}
    A, grads = run(ins, tuple(float(r) for r in g("ranges")), bool(g("meta")[1]), torch.from_numpy(g("G")))
    kind = str(g("type"))
    close(A, g("A").astype(np.float64), f"{kind} A")
    for k, got in grads.items():
        close(got, g(f"d{k}").astype(np.float64), f"{kind} d{k}")


TERMS = [c for r in range(1, 5) for c in itertools.combinations(("M", "R", "dpre", "S"), r)]


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("vec", [False, True])
@pytest.mark.parametrize("terms", TERMS, ids=["+".join(t) for t in TERMS])
def test_matches_oracle(n, vec, terms):
    from oracle import generator as ogen

    gen = torch.Generator().manual_seed(n * 100 + len(terms))
    T, nd = 300, n if vec else 1
    ins = {}
    for k in terms:
        ins[k] = torch.randn(T, n, generator=gen) if k == "dpre" else torch.randn(T, n, n, generator=gen)
    if "M" in terms:
        ins["lc"] = torch.randn(T, nd, generator=gen)
    if any(k in terms for k in ("R", "dpre", "S")):
        ins["ld"] = torch.randn(T, nd, generator=gen)
    G = torch.randn(T, n, n, generator=gen)
    ranges = (0.01, 0.9, 0.02, 0.8)
    A, grads = run(ins, ranges, vec, G)
    ref_in = {k: v.double().requires_grad_(True) for k, v in ins.items()}
    Aref = ogen.generator(**ref_in, ranges=ranges, vec_dt=vec)
    Aref.backward(G.double())
    close(A, Aref.detach().numpy(), "A")
    for k in ins:
        close(grads[k], ref_in[k].grad.numpy(), f"d{k}")


def test_softplus_threshold_and_leading_dims():
    """Pre-activations past softplus's linear threshold (x > 20), and [B, S] leading dims."""
    from hyperconnections_b200.ops import cghc_generator
    from oracle import generator as ogen

    g = torch.Generator().manual_seed(3)
    S = 30.0 * torch.randn(2, 5, 4, 4, generator=g)
    dpre = 30.0 * torch.randn(2, 5, 4, generator=g)
    ld = torch.randn(2, 5, 4, generator=g)
    A = cghc_generator(scores=S.cuda(), diag_pre=dpre.cuda(), logit_diss=ld.cuda(), vec_dt=True)
    assert A.shape == (2, 5, 4, 4)
    ref = ogen.generator(S=S.double(), dpre=dpre.double(), ld=ld.double(), vec_dt=True)
    close(A, ref.numpy(), "A")


def test_errors():
    from hyperconnections_b200.ops import cghc_generator

    with pytest.raises(ValueError):
        cghc_generator(M=torch.randn(2, 4, 4, device="cuda"))  # no logit_conserv
    with pytest.raises(RuntimeError, match="CUDA"):
        cghc_generator(M=torch.randn(2, 4, 4), logit_conserv=torch.randn(2, 1))
    with pytest.raises(RuntimeError, match="n <= 8"):
        cghc_generator(M=torch.randn(2, 9, 9, device="cuda"), logit_conserv=torch.randn(2, 1, device="cuda"))
