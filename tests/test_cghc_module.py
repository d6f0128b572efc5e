"""The CGHC layer of this package against the reference's own layer
(hyperconnections/cghc.py:14-457).

tests/golden/module.npz holds, for seven layers covering every generator
family, the three projection modes, m = 1..4, scalar and per-stream dt,
learn_dt, biased read / write heads and an affine RMSNorm, the reference
layer's state_dict, input, forward output, upstream gradient and the
gradients of the input and every trainable parameter (float32, eager path).

* CPU: the state_dict of hyperconnections_b200.cghc.ContinuousGenHyperConnections
  has exactly the reference's keys and shapes, so a reference checkpoint loads
  with strict=True.
* GPU: with the reference's weights loaded, the layer's output and input
  gradient match the reference's to 1e-5 relative to their largest magnitude
  (float32), and every parameter gradient to 5e-5: those are sums over the
  tokens of chain-rule products through RMSNorm, one GEMM, the generator and
  the matrix exponential (Pade [7/7] here, torch.linalg.matrix_exp there),
  and the dt-head gradients cancel across tokens, so their float32 rounding
  relative to the result is a few times that of the terms (measured up to
  1.1e-5 on a one-element dt bias). Where the reference is installed
  (baseline/_ref) the same holds against the reference layer run on the GPU,
  with bf16 streams as well.
"""

PARAM_TOL = 5e-5

import numpy as np
import pytest
import torch

from tests.conftest import load_golden

MOD = load_golden("module.npz")
CASES = sorted({k.split("/")[0] for k in MOD})
GENS = ["conservative", "psd_diss", "diagonal_diss", "laplacian", "conservative_diag_diss", "conservative_psd_diss",
        "conservative_laplacian"]
PROJS = ["none", "mean", "v"]


def config(case):
    n, m, E, gen, proj, vec_dt, learn_dt, bias, affine = (int(v) for v in MOD[f"{case}/meta"])
    return dict(n=n, m=m, input_dim=n * E // m, embed_dim=E, dt=0.2, generator_type=GENS[gen],
                projection=PROJS[proj], vec_dt=bool(vec_dt), learn_dt=bool(learn_dt), bias=bool(bias),
                elementwise_affine=bool(affine))


def build(case, device="cpu"):
    from hyperconnections_b200.cghc import ContinuousGenHyperConnections

    cfg = config(case)
    E = cfg["embed_dim"]
    layer = ContinuousGenHyperConnections(module=torch.nn.Linear(E, E), **cfg)
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
    grads = {k.split("/", 2)[2] for k in MOD if k.startswith(f"{case}/grad/")}
    assert grads <= {k for k, p in layer.named_parameters() if p.requires_grad}


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
    # the same parameters get gradients as in the reference (an unused head gets none)
    with_grad = {name for name, p in layer.named_parameters() if p.grad is not None}
    assert with_grad == {k.split("/", 2)[2] for k in MOD if k.startswith(f"{case}/grad/")}
    for name in with_grad:
        _close(dict(layer.named_parameters())[name].grad, MOD[f"{case}/grad/{name}"], f"grad {name}", PARAM_TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
def test_layer_matches_reference_layer_on_gpu(case, dtype):
    """Both layers on the GPU with the same weights and input. In bf16 (under
    autocast, as the layers train) the reference rounds Phi and the written
    term Y to bf16 before mixing (cghc.py:321, :417) where this layer keeps
    them in fp32, so there the check is a relative Frobenius error below 2e-2
    on the output and the input gradient."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from baseline import reference_env

    if not reference_env.available():
        pytest.skip("reference not installed in baseline/_ref")
    hc = reference_env.import_reference()
    try:
        cfg = config(case)
        E = cfg["embed_dim"]
        ref = hc.cghc.ContinuousGenHyperConnections(module=torch.nn.Linear(E, E), use_triton=False, **cfg)
        ours, sd = build(case)
        ref.load_state_dict(sd, strict=True)
        ours.load_state_dict(sd, strict=True)
        ref, ours = ref.cuda(), ours.cuda()
        torch.manual_seed(3)
        x = torch.randn(4, 9, cfg["input_dim"], device="cuda").to(dtype)
        g = torch.randn_like(x)
        res = []
        for layer in (ref, ours):
            xi = x.clone().requires_grad_(True)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
                out = layer(xi)
            out.backward(g)
            res.append((out, xi.grad, {k: p.grad for k, p in layer.named_parameters() if p.grad is not None}))
        (o_r, gx_r, p_r), (o_o, gx_o, p_o) = res
        if dtype == torch.float32:
            _close(o_o, o_r.detach().double().cpu().numpy(), "out")
            _close(gx_o, gx_r.double().cpu().numpy(), "grad_x")
            for k in p_r:
                _close(p_o[k], p_r[k].double().cpu().numpy(), f"grad {k}", PARAM_TOL)
        else:
            assert o_o.dtype == o_r.dtype == torch.bfloat16
            for a, b, what in ((o_o, o_r, "out"), (gx_o, gx_r, "grad_x")):
                rel = ((a.double() - b.double()).norm() / b.double().norm()).item()
                assert rel < 2e-2, f"bf16 {what}: relative error {rel:.3e}"
            assert p_r.keys() == p_o.keys()
    finally:
        reference_env._forget_reference()
