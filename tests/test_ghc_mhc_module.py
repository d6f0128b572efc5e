"""The GHC and MHC layers of this package against the reference's own layers
(hyperconnections/ghc.py:14-128, mhc.py:21-150).

tests/golden/module_ghc_mhc.npz holds five layers of each (n, m up to 8, 4;
biased heads; affine RMSNorm; 0, 7 and 20 Sinkhorn iterations), wrapping a
Linear, with every parameter moved off its init: the state_dict, input,
forward output, upstream gradient and the gradients of the input and every
parameter (float32, the reference's eager code).

* CPU: this package's layers have exactly the reference's state_dict keys
  and shapes (a reference checkpoint loads with strict=True).
* GPU: output and input gradient to 1e-5 relative to their largest
  magnitude, parameter gradients (sums over the tokens through RMSNorm, one
  GEMM and, for MHC, the Sinkhorn projection) to 5e-5; the same against the
  installed reference run on the GPU (baseline/_ref).
"""

import numpy as np
import pytest
import torch

from tests.conftest import load_golden

MOD = load_golden("module_ghc_mhc.npz")
CASES = sorted({k.split("/")[0] for k in MOD})
PARAM_TOL = 5e-5


def build(case, ref_module=None):
    meta = [int(v) for v in MOD[f"{case}/meta"]]
    n, m, E, bias, affine = meta[:5]
    kw = dict(bias=bool(bias), elementwise_affine=bool(affine))
    if case.startswith("m"):
        kw["sinkhorn_iters"] = meta[5]
    if ref_module is None:
        from hyperconnections_b200.ghc import GeneralizedHyperConnections as GHC
        from hyperconnections_b200.mhc import ManifoldHyperConnections as MHC
    else:
        GHC, MHC = ref_module.ghc.GeneralizedHyperConnections, ref_module.mhc.ManifoldHyperConnections
    cls = MHC if case.startswith("m") else GHC
    layer = cls(n, m, n * E // m, E, torch.nn.Linear(E, E), **kw)
    sd = {k.split("/", 2)[2]: torch.from_numpy(MOD[k]) for k in MOD if k.startswith(f"{case}/sd/")}
    return layer, sd


@pytest.mark.parametrize("case", CASES)
def test_state_dict_matches_reference(case):
    layer, sd = build(case)
    ours = layer.state_dict()
    assert sorted(ours) == sorted(sd)
    for k in sd:
        assert tuple(ours[k].shape) == tuple(sd[k].shape), k
    layer.load_state_dict(sd, strict=True)


def _close(got, ref, what, tol=1e-5):
    got = got.detach().double().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    bound = tol * max(1.0, np.abs(ref).max())
    assert err <= bound, f"{what}: max err {err:.3e} > {bound:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_layer_matches_reference_fixture(case):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    layer, sd = build(case)
    layer.load_state_dict(sd, strict=True)
    layer = layer.cuda()
    x = torch.from_numpy(MOD[f"{case}/x"]).cuda().requires_grad_(True)
    out = layer(x)
    out.backward(torch.from_numpy(MOD[f"{case}/g"]).cuda())
    _close(out, MOD[f"{case}/out"], "out")
    _close(x.grad, MOD[f"{case}/grad_x"], "grad_x")
    with_grad = {name for name, p in layer.named_parameters() if p.grad is not None}
    assert with_grad == {k.split("/", 2)[2] for k in MOD if k.startswith(f"{case}/grad/")}
    params = dict(layer.named_parameters())
    for name in with_grad:
        _close(params[name].grad, MOD[f"{case}/grad/{name}"], f"grad {name}", PARAM_TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_layer_matches_reference_layer_on_gpu(case):
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from baseline import reference_env

    if not reference_env.available():
        pytest.skip("reference not installed in baseline/_ref")
    hc = reference_env.import_reference()
    try:
        ref, sd = build(case, hc)
        ours, _ = build(case)
        ref.load_state_dict(sd, strict=True)
        ours.load_state_dict(sd, strict=True)
        ref, ours = ref.cuda(), ours.cuda()
        torch.manual_seed(5)
        x = torch.randn(3, 11, ref.input_dim, device="cuda")
        g = torch.randn_like(x)
        res = []
        for layer in (ref, ours):
            xi = x.clone().requires_grad_(True)
            out = layer(xi)
            out.backward(g)
            res.append((out.detach(), xi.grad, {k: p.grad for k, p in layer.named_parameters() if p.grad is not None}))
        (o_r, gx_r, p_r), (o_o, gx_o, p_o) = res
        _close(o_o, o_r.double().cpu().numpy(), "out")
        _close(gx_o, gx_r.double().cpu().numpy(), "grad_x")
        assert p_r.keys() == p_o.keys()
        for k in p_r:
            _close(p_o[k], p_r[k].double().cpu().numpy(), f"grad {k}", PARAM_TOL)
    finally:
        reference_env._forget_reference()
