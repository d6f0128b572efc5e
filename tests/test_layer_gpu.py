"""GPU parity of one hyper-connection layer built from the kernels, against
the reference's own CGHC layer (hyperconnections/cghc.py).

The fixtures (tests/golden/layer.npz) hold, for six layers covering every
generator family and projection mode, the reference layer's read / write
weights, generator A, projection direction and forward output, and the
gradients of its chain read (:410) -> wrapped Linear -> write (:417) ->
matrix_exp (:321) -> mix (:449). Here the same chain runs as
matrix_exp -> hc_read -> Linear -> hc_mix_write on the GPU in float32;
outputs and every gradient must agree to 1e-5 relative to their largest
magnitude (the fixtures' own float32 error is at most 2.6e-6).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

LAYER = load_golden("layer.npz")
CASES = sorted({k.split("_")[0] for k in LAYER})


@pytest.fixture(autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")


@pytest.mark.parametrize("case", CASES)
def test_cghc_layer_chain_matches_reference(case):
    from hyperconnections_b200.ops import hc_mix_write, hc_read, matrix_exp

    g = lambda name: torch.from_numpy(LAYER[f"{case}_{name}"]).cuda()  # noqa: E731
    n, m, E, block, T, has_v = (int(v) for v in LAYER[f"{case}_meta"])
    leaves = {k: g(k).clone().requires_grad_(True) for k in ("x", "read_in", "write_out", "A", "W_mod", "b_mod")}
    if has_v:
        leaves["v"] = g("v").clone().requires_grad_(True)
    Phi = matrix_exp(leaves["A"])
    u = hc_read(leaves["read_in"], leaves["x"])
    f = F.linear(u.reshape(T, m * block), leaves["W_mod"], leaves["b_mod"]).reshape(T, m, block)
    out = hc_mix_write(Phi, leaves["x"], leaves["write_out"], f, leaves.get("v"))
    out.backward(g("g"))

    def close(got, name):
        ref = LAYER[f"{case}_{name}"].astype(np.float64)
        err = np.abs(got.detach().double().cpu().numpy() - ref).max()
        bound = 1e-5 * max(1.0, np.abs(ref).max())
        assert err <= bound, f"{name}: max err {err:.3e} > {bound:.3e}"

    close(out, "out")
    for k in leaves:
        close(leaves[k].grad, f"grad_{k}")
