"""Generate the golden fixtures of tests/golden/ by running the REFERENCE's own
code (pjjajal/hyperconnections) on the CPU of this container.

    python tests/golden/make_golden.py --reference <checkout of pjjajal/hyperconnections>

(or set HC_REFERENCE to that checkout's root)

What runs, all from the reference checkout, unmodified:
  * expm_t18's Python body (hyperconnections/ops/expm.py:65-106) without its
    torch.compile wrapper (the compiled form does not build on this CPU), with
    autograd for the gradient -> expm_t18.npz;
  * torch.linalg.matrix_exp, which CGHC calls (cghc.py:321) -> matrix_exp.npz;
  * the reference's Triton stream-mix kernels and autograd Function
    (ops/stream_mix_small_nb.py) under TRITON_INTERPRET=1 with a fixed BLOCK_D
    (the autotuner needs a GPU) -> stream_mix_*.npz (N = 1..32);
  * CGHC's composition read einsum (cghc.py:410) -> write einsum (:417) ->
    stream_mix_add (:449, the small-NB Function) in float32 on bf16-exact
    inputs, forward and backward -> fused.npz;
  * the same composition for m backbone blocks with the reference's own
    einops patterns, with and without the projection direction -> rw.npz;
  * one CGHC layer (cghc.py) per generator type and projection mode: its own
    read/write weights, generator, projection and forward output, with the
    gradients of its read -> module -> write -> matrix_exp -> mix chain
    -> layer.npz;
  * MHC's Sinkhorn-Knopp method (mhc.py:97-102) with autograd -> sinkhorn.npz;
  * CGHC's compute_generator (cghc.py:219-315) for every generator type and
    dt mode, its Linear outputs captured by hooks -> generator.npz.

The reference imports timm only for trunc_normal_; a stub providing
torch.nn.init.trunc_normal_ is written to a temporary directory and put on
sys.path. Nothing else is patched. Inputs follow the reference tests' seeds
(tests/test_ops.py:48-63) and the benchmark's structured-Phi families
(benchmarks/stream_mix_bench.py:93-120).
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path: str):
    stub = tempfile.mkdtemp(prefix="timm_stub_")
    os.makedirs(os.path.join(stub, "timm", "models"))
    open(os.path.join(stub, "timm", "__init__.py"), "w").close()
    open(os.path.join(stub, "timm", "models", "__init__.py"), "w").close()
    with open(os.path.join(stub, "timm", "models", "layers.py"), "w") as fh:
        fh.write("from torch.nn.init import trunc_normal_\n")
    sys.path[:0] = [stub, path]
    import hyperconnections.ops.expm as ref_expm
    import hyperconnections.ops.stream_mix_small_nb as ref_small

    return ref_expm, ref_small


class _FixedBlock:
    """Stands in for an autotuned Triton kernel: launches the inner JIT
    function with one BLOCK_D (the interpreter cannot benchmark configs)."""

    def __init__(self, autotuned, block_d):
        self.fn = autotuned.fn
        self.block_d = block_d

    def __getitem__(self, grid):
        meta = {"BLOCK_D": self.block_d}
        g = grid(meta) if callable(grid) else grid

        def launch(*args, **kwargs):
            return self.fn[g](*args, BLOCK_D=self.block_d, **kwargs)

        return launch


def gen_expm(ref_expm, out):
    body = ref_expm.expm_t18._torchdynamo_orig_callable
    rec = {}
    for n in (1, 2, 3, 4, 6, 8):
        for kind in ("skew", "small", "scaled"):
            g = torch.Generator().manual_seed(1000 + 10 * n + {"skew": 0, "small": 1, "scaled": 2}[kind])
            B = 40
            M = torch.randn(B, n, n, generator=g)
            if kind == "skew":  # the config's distribution: 0.5 * (G - G^T) / 2
                A = 0.5 * (M - M.mT) / 2
            elif kind == "small":  # norms below theta_18: no scaling
                A = 0.3 * M / n
            else:  # norms above theta_18, mixed within the batch (s up to 3)
                A = M * torch.linspace(0.5, 6.0, B).view(B, 1, 1) / n**0.5
            Gr = torch.randn(B, n, n, generator=g)
            A = A.float()
            Ar = A.clone().requires_grad_(True)
            E = body(Ar)
            E.backward(Gr)
            Am = A.clone().requires_grad_(True)
            Em = torch.linalg.matrix_exp(Am)
            Em.backward(Gr)
            key = f"n{n}_{kind}"
            rec[f"{key}_A"] = A.numpy()
            rec[f"{key}_G"] = Gr.numpy()
            rec[f"{key}_E"] = E.detach().numpy()
            rec[f"{key}_dA"] = Ar.grad.numpy()
            rec[f"{key}_Em"] = Em.detach().numpy()
            rec[f"{key}_dAm"] = Am.grad.numpy()
    np.savez_compressed(os.path.join(out, "expm.npz"), **rec)


def _make_inputs(B, N, D, dtype, seed=0):  # reference tests/test_ops.py:48-57
    torch.manual_seed(seed)
    Phi = torch.randn(B, N, N, dtype=dtype)
    x = torch.randn(B, N, D, dtype=dtype)
    Y = torch.randn(B, N, D, dtype=dtype)
    return Phi, x, Y


def _make_v(B, N, dtype, seed=7):  # reference tests/test_ops.py:60-63
    torch.manual_seed(seed)
    return torch.nn.functional.normalize(torch.randn(B, N, dtype=dtype), dim=-1)


def _structured_phi(kind, B, N, dtype):  # reference benchmarks/stream_mix_bench.py:93-111
    if kind == "skew":
        torch.manual_seed(1)
        M = torch.randn(B, N, N, dtype=dtype) / N**0.5
        return (M - M.mT).contiguous()
    if kind == "psd":
        torch.manual_seed(2)
        R = torch.randn(B, N, N, dtype=dtype) / N**0.5
        return (R @ R.mT).contiguous()
    torch.manual_seed(3)
    return torch.diag_embed(torch.randn(B, N, dtype=dtype)).contiguous()


def gen_stream_mix(ref_small, out):
    ref_small._stream_mix_fwd = _FixedBlock(ref_small._stream_mix_fwd, 32)
    ref_small._stream_mix_bwd_dx = _FixedBlock(ref_small._stream_mix_bwd_dx, 32)
    ref_small._stream_mix_bwd_dPhi = _FixedBlock(ref_small._stream_mix_bwd_dPhi, 64)
    fn = ref_small.stream_mix_add_small_nb

    cases = [  # (B, N, D, proj, phi kind) — the shapes of tests/test_ops.py
        (1, 4, 64, False, "random"), (2, 8, 128, False, "random"), (4, 4, 256, False, "random"),
        (3, 6, 48, False, "random"), (1, 4, 64, True, "random"), (2, 8, 128, True, "random"),
        (3, 4, 48, True, "random"), (1, 4, 1, False, "random"), (1, 4, 7, False, "random"),
        (1, 4, 33, False, "random"), (1, 4, 100, False, "random"), (3, 1, 64, False, "random"),
        (2, 3, 40, True, "random"), (2, 5, 24, True, "random"), (1, 7, 16, True, "random"),
        (2, 4, 64, True, "skew"), (2, 4, 64, True, "psd"), (2, 4, 64, True, "diag"),
        (2, 2, 100, True, "random"),
    ]
    rec = {}
    for ci, (B, N, D, proj, kind) in enumerate(cases):
        Phi, x, Y = _make_inputs(B, N, D, torch.float32)
        if kind != "random":
            Phi = _structured_phi(kind, B, N, torch.float32)
        v = _make_v(B, N, torch.float32) if proj else None
        g = torch.Generator().manual_seed(500 + ci)
        Gup = torch.randn(B, N, D, generator=g)
        P = Phi.clone().requires_grad_(True)
        X = x.clone().requires_grad_(True)
        Yr = Y.clone().requires_grad_(True)
        Vr = v.clone().requires_grad_(True) if proj else None
        o = fn(P, X, Yr, Vr)
        o.backward(Gup)
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([B, N, D, int(proj)])
        rec[f"{key}_Phi"] = Phi.numpy()
        rec[f"{key}_x"] = x.numpy()
        rec[f"{key}_Y"] = Y.numpy()
        rec[f"{key}_Gup"] = Gup.numpy()
        rec[f"{key}_out"] = o.detach().numpy()
        rec[f"{key}_gPhi"] = P.grad.numpy()
        rec[f"{key}_gx"] = X.grad.numpy()
        rec[f"{key}_gY"] = Yr.grad.numpy()
        if proj:
            rec[f"{key}_v"] = v.numpy()
            rec[f"{key}_gv"] = Vr.grad.numpy()
    np.savez_compressed(os.path.join(out, "stream_mix_f32.npz"), **rec)

    # fp16 forward (reference tests/test_ops.py:106-112 compares fp16 output
    # against the fp32 bmm of the same fp16 values)
    rec16 = {}
    for ci, (B, N, D) in enumerate([(2, 4, 128), (1, 8, 64), (2, 3, 40)]):
        Phi, x, Y = _make_inputs(B, N, D, torch.float16)
        o = fn(Phi, x, Y, None)
        key = f"c{ci}"
        rec16[f"{key}_Phi"] = Phi.numpy()
        rec16[f"{key}_x"] = x.numpy()
        rec16[f"{key}_Y"] = Y.numpy()
        rec16[f"{key}_out"] = o.numpy()
    np.savez_compressed(os.path.join(out, "stream_mix_f16.npz"), **rec16)


def gen_stream_mix_large_n(ref_small, out):
    """stream_mix_add at 9 <= N <= 32 through the reference's small-NB Function
    (the kernel stream_mix_add runs below the big-NB size threshold,
    ops/stream_mix.py:45-51), float32, with and without projection."""
    fn = ref_small.stream_mix_add_small_nb
    cases = [(2, 12, 40, False), (2, 12, 40, True), (1, 16, 96, False), (2, 16, 33, True), (1, 32, 64, True),
             (1, 9, 17, False), (1, 24, 48, True)]
    rec = {}
    for ci, (B, N, D, proj) in enumerate(cases):
        Phi, x, Y = _make_inputs(B, N, D, torch.float32, seed=6000 + ci)
        v = _make_v(B, N, torch.float32, seed=6100 + ci) if proj else None
        g = torch.Generator().manual_seed(6200 + ci)
        Gup = torch.randn(B, N, D, generator=g)
        P, X, Yr = (t.clone().requires_grad_(True) for t in (Phi, x, Y))
        Vr = v.clone().requires_grad_(True) if proj else None
        o = fn(P, X, Yr, Vr)
        o.backward(Gup)
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([B, N, D, int(proj)])
        items = [("Phi", Phi), ("x", x), ("Y", Y), ("Gup", Gup), ("out", o.detach()), ("gPhi", P.grad), ("gx", X.grad)]
        if proj:
            items += [("v", v), ("gv", Vr.grad)]
        for name, t in items:
            rec[f"{key}_{name}"] = t.numpy()
    np.savez_compressed(os.path.join(out, "stream_mix_large_n.npz"), **rec)


def gen_fused(ref_small, out):
    """CGHC composition (cghc.py:410, :417, :449) with m = 1, float32 math on
    bf16-exact inputs drawn like the fused-step workload."""
    fn = ref_small.stream_mix_add_small_nb
    rec = {}
    for ci, (T, n, D) in enumerate([(32, 4, 96), (24, 2, 64), (16, 3, 40), (16, 6, 48), (12, 8, 72), (8, 4, 100)]):
        g = torch.Generator().manual_seed(2000 + ci)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).float()  # noqa: E731
        x = bf(T, n, D)
        f = bf(T, D)
        S = torch.triu(0.5 * torch.randn(T, n, n, generator=g), 1)
        H = torch.linalg.matrix_exp(S - S.mT)
        alpha = torch.softmax(torch.randn(T, n, generator=g), -1)
        beta = torch.softmax(torch.randn(T, n, generator=g), -1)
        g_u = bf(T, D)
        g_x = bf(T, n, D)
        X, Fv, Hr, Ar, Br = (t.clone().requires_grad_(True) for t in (x, f, H, alpha, beta))
        read_in = Ar[:, None, :]    # [T, m=1, n]
        write_out = Br[:, :, None]  # [T, n, m=1]
        u = torch.einsum("bmn,bnd->bmd", read_in, X)          # cghc.py:410
        Y = torch.einsum("bnm,bmd->bnd", write_out, Fv[:, None, :])  # cghc.py:417
        x_out = fn(Hr, X, Y, None)                              # cghc.py:449 -> :363
        torch.autograd.backward([u, x_out], [g_u[:, None, :], g_x])
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([T, n, D])
        for name, t in (("x", x), ("f", f), ("H", H), ("alpha", alpha), ("beta", beta), ("g_u", g_u),
                        ("g_x", g_x), ("u", u[:, 0].detach()), ("x_out", x_out.detach()),
                        ("grad_x", X.grad), ("grad_f", Fv.grad), ("grad_H", Hr.grad),
                        ("grad_alpha", Ar.grad), ("grad_beta", Br.grad)):
            rec[f"{key}_{name}"] = t.numpy()
    np.savez_compressed(os.path.join(out, "fused.npz"), **rec)


def gen_rw(ref_small, out):
    """Read einsum (cghc.py:410) and write einsum (:417) with the reference's
    own einops patterns, then the mix through stream_mix_add (:449), for
    general m, with and without the projection direction; float32 math on
    bf16-exact inputs. Shapes include the reference test CONFIGS
    (tests/test_cghc.py:21-26, test_ghc.py:22-29: (n, m, embed_dim) with
    block size embed_dim / m) and 16-byte-aligned block sizes."""
    from einops import einsum

    fn = ref_small.stream_mix_add_small_nb
    cases = [  # (T, n, m, D, proj)
        (6, 2, 1, 8, False), (6, 4, 2, 4, False), (5, 4, 4, 2, True), (4, 6, 3, 4, False), (6, 2, 2, 4, True),
        (16, 4, 2, 64, True), (8, 8, 4, 128, False), (12, 3, 3, 40, True), (10, 6, 2, 48, False),
        (6, 2, 2, 100, True), (20, 4, 1, 96, True), (9, 8, 1, 64, True), (7, 5, 4, 72, True),
    ]
    rec = {}
    for ci, (T, n, m, D, proj) in enumerate(cases):
        g = torch.Generator().manual_seed(3000 + ci)
        bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).float()  # noqa: E731
        x = bf(T, n, D)
        f = bf(T, m, D)
        R = torch.sigmoid(torch.randn(T, m, n, generator=g))          # read_in  [B, m, n]
        W = 2 * torch.sigmoid(torch.randn(T, n, m, generator=g))      # write_out [B, n, m]
        S = torch.triu(0.5 * torch.randn(T, n, n, generator=g), 1)
        H = torch.linalg.matrix_exp(S - S.mT)
        v = torch.nn.functional.normalize(torch.randn(T, n, generator=g), dim=-1) if proj else None
        g_u = bf(T, m, D)
        g_x = bf(T, n, D)
        X, Fv, Rr, Wr, Hr = (t.clone().requires_grad_(True) for t in (x, f, R, W, H))
        Vr = v.clone().requires_grad_(True) if proj else None
        u = einsum(Rr, X, "b m n, b n d -> b m d")                     # cghc.py:410
        Y = einsum(Wr, Fv, "b n m, b m d -> b n d")                    # cghc.py:417
        x_out = fn(Hr, X, Y, Vr)                                       # cghc.py:449 -> :363
        torch.autograd.backward([u, x_out], [g_u, g_x])
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([T, n, m, D, int(proj)])
        items = [("x", x), ("f", f), ("R", R), ("W", W), ("H", H), ("g_u", g_u), ("g_x", g_x),
                 ("u", u.detach()), ("x_out", x_out.detach()), ("grad_x", X.grad), ("grad_f", Fv.grad),
                 ("grad_R", Rr.grad), ("grad_W", Wr.grad), ("grad_H", Hr.grad)]
        if proj:
            items += [("v", v), ("grad_v", Vr.grad)]
        for name, t in items:
            rec[f"{key}_{name}"] = t.numpy()
    np.savez_compressed(os.path.join(out, "rw.npz"), **rec)


def gen_layer(ref_path, out):
    """One CGHC layer of the reference (hyperconnections/cghc.py), eager path,
    float32: its own read/write weights (:323-339), generator (:219-315) and
    projection (:341-350) for a seeded input, the layer's own forward output,
    and the gradients of the chain read (:410) -> module -> write (:417) ->
    matrix_exp (:321) -> mix (:449) with respect to x, the weights, the
    generator, the projection direction and the wrapped Linear's parameters.
    The chain is checked against the layer's forward before it is saved."""
    from einops import einsum
    from hyperconnections.cghc import ContinuousGenHyperConnections as CGHC

    configs = [  # (n, m, embed_dim, generator_type, projection, vec_dt)
        (4, 1, 64, "conservative_psd_diss", "none", False),
        (4, 2, 128, "conservative_diag_diss", "mean", False),
        (6, 3, 96, "conservative_laplacian", "v", True),
        (2, 1, 8, "conservative", "none", False),
        (4, 4, 8, "psd_diss", "v", False),
        (8, 2, 128, "laplacian", "mean", True),
    ]
    rec = {}
    for ci, (n, m, E, gen, proj, vec_dt) in enumerate(configs):
        torch.manual_seed(4000 + ci)
        block = E // m
        inp = n * block
        module = torch.nn.Linear(E, E)
        layer = CGHC(n, m, inp, E, module, dt=0.3, generator_type=gen, projection=proj, vec_dt=vec_dt,
                     use_triton=False)
        with torch.no_grad():  # move the static parameters off their init values
            for name, prm in layer.named_parameters():
                if not name.startswith("module.") and prm.dim() >= 1:
                    prm.add_(0.3 * torch.randn_like(prm))
        B, S = 2, 5
        x = torch.randn(B, S, inp).to(torch.bfloat16).float()
        g = torch.randn(B, S, inp)
        with torch.no_grad():
            ref_out = layer(x)
        xf = x.reshape(-1, n, block)
        with torch.no_grad():
            write_out, read_in = layer.compute_read_write_weights(xf)
            A = layer.compute_generator(xf)
            v = layer.compute_projection(xf)
        X, RI, WO, AL = (t.detach().clone().requires_grad_(True) for t in (xf, read_in, write_out, A))
        V = None if v is None else v.detach().clone().requires_grad_(True)
        u = einsum(RI, X, "b m n, b n d -> b m d")                              # cghc.py:410
        f = layer.module(u.reshape(B, S, E)).reshape(-1, m, block)
        Y = einsum(WO, f, "b n m, b m d -> b n d")                             # cghc.py:417
        Phi = torch.linalg.matrix_exp(AL.float()).to(x.dtype)                  # cghc.py:321
        outc = layer._stream_mix(X, Phi, Y, V)                                   # cghc.py:449
        assert torch.allclose(outc.reshape(B, S, inp), ref_out, rtol=1e-6, atol=1e-6)
        layer.zero_grad()
        outc.backward(g.reshape(-1, n, block))
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([n, m, E, block, B * S, int(V is not None)])
        items = [("x", xf), ("read_in", read_in), ("write_out", write_out), ("A", A), ("g", g.reshape(-1, n, block)),
                 ("W_mod", module.weight.detach()), ("b_mod", module.bias.detach()), ("out", ref_out.reshape(-1, n, block)),
                 ("grad_x", X.grad), ("grad_read_in", RI.grad), ("grad_write_out", WO.grad), ("grad_A", AL.grad),
                 ("grad_W_mod", module.weight.grad), ("grad_b_mod", module.bias.grad)]
        if V is not None:
            items += [("v", v), ("grad_v", V.grad)]
        for name, t in items:
            rec[f"{key}_{name}"] = t.detach().numpy()
    np.savez_compressed(os.path.join(out, "layer.npz"), **rec)


def gen_module(out):
    """Whole CGHC layers of the reference (hyperconnections/cghc.py:14-457),
    eager path, float32, wrapping a Linear: the layer's state_dict (its own
    parameter names), a seeded input, the forward output, an upstream
    gradient and the gradient of the input and of every trainable parameter.
    Covers every generator family, the three projection modes, m = 1..4,
    scalar and per-stream dt, learn_dt, biased heads and an affine RMSNorm.
    Keys: "<case>/meta", "<case>/x", "<case>/g", "<case>/out", "<case>/grad_x",
    "<case>/sd/<name>", "<case>/grad/<name>"."""
    from hyperconnections.cghc import ContinuousGenHyperConnections as CGHC

    configs = [  # (n, m, embed_dim, generator_type, projection, vec_dt, learn_dt, bias, affine)
        (4, 1, 64, "conservative_psd_diss", "none", False, False, False, False),
        (4, 2, 128, "conservative_diag_diss", "mean", False, False, False, False),
        (6, 3, 96, "conservative_laplacian", "v", True, True, False, False),
        (2, 1, 32, "conservative", "none", False, False, True, True),
        (4, 4, 32, "psd_diss", "v", False, True, True, False),
        (8, 2, 128, "laplacian", "mean", True, False, False, True),
        (3, 1, 48, "diagonal_diss", "none", True, True, False, False),
    ]
    gen_codes = ["conservative", "psd_diss", "diagonal_diss", "laplacian", "conservative_diag_diss",
                 "conservative_psd_diss", "conservative_laplacian"]
    proj_codes = ["none", "mean", "v"]
    rec = {}
    for ci, (n, m, E, gen, proj, vec_dt, learn_dt, bias, affine) in enumerate(configs):
        torch.manual_seed(5000 + ci)
        inp = n * E // m
        layer = CGHC(n, m, inp, E, torch.nn.Linear(E, E), dt=0.2, generator_type=gen, projection=proj,
                     learn_dt=learn_dt, bias=bias, elementwise_affine=affine, use_triton=False, vec_dt=vec_dt)
        with torch.no_grad():  # move every parameter off its init value
            for prm in layer.parameters():
                prm.add_(0.3 * torch.randn_like(prm))
            if proj == "mean":
                layer.projection_dir.add_(0.2 * torch.randn_like(layer.projection_dir))
                layer.projection_dir.div_(layer.projection_dir.norm())
        x = torch.randn(2, 5, inp, requires_grad=True)
        g = torch.randn(2, 5, inp)
        y = layer(x)
        y.backward(g)
        key = f"c{ci}"
        rec[f"{key}/meta"] = np.array([n, m, E, gen_codes.index(gen), proj_codes.index(proj), int(vec_dt),
                                       int(learn_dt), int(bias), int(affine)])
        rec[f"{key}/x"] = x.detach().numpy()
        rec[f"{key}/g"] = g.numpy()
        rec[f"{key}/out"] = y.detach().numpy()
        rec[f"{key}/grad_x"] = x.grad.numpy()
        for name, t in layer.state_dict().items():
            rec[f"{key}/sd/{name}"] = t.detach().numpy()
        for name, prm in layer.named_parameters():
            if prm.grad is not None:
                rec[f"{key}/grad/{name}"] = prm.grad.numpy()
    np.savez_compressed(os.path.join(out, "module.npz"), **rec)


def _record_layer(rec, key, layer, inp, seed, meta):
    """One layer's state_dict, input, output, upstream gradient and the
    gradients of the input and every parameter that gets one."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, 5, inp, generator=g).requires_grad_(True)
    up = torch.randn(2, 5, inp, generator=g)
    y = layer(x)
    y.backward(up)
    rec[f"{key}/meta"] = np.array(meta)
    rec[f"{key}/x"] = x.detach().numpy()
    rec[f"{key}/g"] = up.numpy()
    rec[f"{key}/out"] = y.detach().numpy()
    rec[f"{key}/grad_x"] = x.grad.numpy()
    for name, t in layer.state_dict().items():
        rec[f"{key}/sd/{name}"] = t.detach().numpy()
    for name, prm in layer.named_parameters():
        if prm.grad is not None:
            rec[f"{key}/grad/{name}"] = prm.grad.numpy()


def gen_module_ghc_mhc(out):
    """Whole GHC (hyperconnections/ghc.py:14-128) and MHC (mhc.py:21-150)
    layers of the reference, float32, wrapping a Linear, with every parameter
    moved off its init value: the same record as gen_module ("g<i>/...",
    "m<i>/..."; meta = n, m, embed_dim, bias, affine[, sinkhorn iters])."""
    from hyperconnections.ghc import GeneralizedHyperConnections as GHC
    from hyperconnections.mhc import ManifoldHyperConnections as MHC

    rec = {}
    ghc_cfgs = [(4, 1, 64, False, False), (4, 2, 128, True, False), (6, 3, 96, False, True), (2, 2, 32, False, False),
                (8, 4, 128, True, True)]
    for ci, (n, m, E, bias, affine) in enumerate(ghc_cfgs):
        torch.manual_seed(6000 + ci)
        layer = GHC(n, m, n * E // m, E, torch.nn.Linear(E, E), bias=bias, elementwise_affine=affine)
        with torch.no_grad():
            for prm in layer.parameters():
                prm.add_(0.3 * torch.randn_like(prm))
        _record_layer(rec, f"g{ci}", layer, n * E // m, 6100 + ci, [n, m, E, int(bias), int(affine)])
    mhc_cfgs = [(4, 1, 64, False, False, 20), (4, 2, 128, True, False, 20), (6, 3, 96, False, True, 7),
                (2, 1, 32, False, False, 0), (8, 4, 128, True, True, 20)]
    for ci, (n, m, E, bias, affine, iters) in enumerate(mhc_cfgs):
        torch.manual_seed(7000 + ci)
        layer = MHC(n, m, n * E // m, E, torch.nn.Linear(E, E), bias=bias, elementwise_affine=affine,
                    sinkhorn_iters=iters)
        with torch.no_grad():
            for prm in layer.parameters():
                prm.add_(0.3 * torch.randn_like(prm))
        _record_layer(rec, f"m{ci}", layer, n * E // m, 7100 + ci, [n, m, E, int(bias), int(affine), iters])
    np.savez_compressed(os.path.join(out, "module_ghc_mhc.npz"), **rec)


def gen_generator(out):
    """CGHC's generator (cghc.py:219-315) for every generator type, scalar and
    per-stream dt, computed by the reference layer's own compute_generator
    with autograd. Forward hooks capture its Linear outputs; the fixture
    stores the pre-activations the kernel takes (static parameter + Linear
    output), the generator A, an upstream gradient and the gradients of the
    Linear outputs (equal to those of the pre-activations)."""
    from hyperconnections.cghc import ContinuousGenHyperConnections as CGHC

    types = ["conservative", "psd_diss", "diagonal_diss", "laplacian", "conservative_diag_diss",
             "conservative_psd_diss", "conservative_laplacian"]
    configs = [(4, t, v) for t in types for v in (False, True)] + [(2, "conservative_psd_diss", True),
                                                                   (6, "conservative_laplacian", False),
                                                                   (8, "conservative_psd_diss", True),
                                                                   (3, "conservative_diag_diss", True)]
    rec = {}
    for ci, (n, gen, vec) in enumerate(configs):
        torch.manual_seed(7000 + ci)
        block, m = 8, 1
        layer = CGHC(n, m, n * block, m * block, torch.nn.Identity(), dt=0.3, generator_type=gen, vec_dt=vec,
                     use_triton=False)
        with torch.no_grad():
            for name, prm in layer.named_parameters():
                if prm.dim() >= 1:
                    prm.add_(0.5 * torch.randn_like(prm))
        captured = {}

        def hook(name):
            def fn(_mod, _inp, outp):
                outp.retain_grad()
                captured[name] = outp
            return fn

        for name in ("conv_pred", "dt_proj_conserv", "dt_proj_diss", "diss_pred", "laplacian_pred"):
            if hasattr(layer, name):
                getattr(layer, name).register_forward_hook(hook(name))
        T = 20
        x = torch.randn(T, n, block)
        A = layer.compute_generator(x)
        G = torch.randn(T, n, n)
        A.backward(G)
        key = f"c{ci}"
        has_diss = any(hasattr(layer, k) for k in ("diss_A", "diss_diag", "laplacian_A"))
        rec[f"{key}_meta"] = np.array([n, int(vec), T])
        rec[f"{key}_type"] = np.array(gen)
        rec[f"{key}_ranges"] = np.array([layer.dt_min_cons, layer.dt_max_cons, layer.dt_min_diss, layer.dt_max_diss])
        rec[f"{key}_A"] = A.detach().numpy()
        rec[f"{key}_G"] = G.numpy()
        with torch.no_grad():
            if hasattr(layer, "conserv_A"):
                rec[f"{key}_M"] = (layer.conserv_A + captured["conv_pred"].reshape(T, n, n)).numpy()
                rec[f"{key}_dM"] = captured["conv_pred"].grad.reshape(T, n, n).numpy()
                rec[f"{key}_lc"] = (layer.log_dt_conserv + captured["dt_proj_conserv"]).numpy()
                rec[f"{key}_dlc"] = captured["dt_proj_conserv"].grad.numpy()
            if has_diss:
                rec[f"{key}_ld"] = (layer.log_dt_diss + captured["dt_proj_diss"]).numpy()
                rec[f"{key}_dld"] = captured["dt_proj_diss"].grad.numpy()
            if hasattr(layer, "diss_A"):
                rec[f"{key}_R"] = (layer.diss_A + captured["diss_pred"].reshape(T, n, n)).numpy()
                rec[f"{key}_dR"] = captured["diss_pred"].grad.reshape(T, n, n).numpy()
            if hasattr(layer, "diss_diag"):
                rec[f"{key}_dpre"] = (layer.diss_diag + captured["diss_pred"]).numpy()
                rec[f"{key}_ddpre"] = captured["diss_pred"].grad.numpy()
            if hasattr(layer, "laplacian_A"):
                rec[f"{key}_S"] = (layer.laplacian_A + captured["laplacian_pred"].reshape(T, n, n)).numpy()
                rec[f"{key}_dS"] = captured["laplacian_pred"].grad.reshape(T, n, n).numpy()
    np.savez_compressed(os.path.join(out, "generator.npz"), **rec)


def gen_sinkhorn(out):
    """MHC's Sinkhorn-Knopp projection (mhc.py:97-102) run as the reference's
    own method, float32, with autograd for the gradient."""
    from types import SimpleNamespace

    from hyperconnections.mhc import ManifoldHyperConnections as MHC

    rec = {}
    cases = [(64, 4, 20, 0.0), (37, 2, 20, 1.0), (50, 3, 5, 0.5), (16, 6, 20, 1.0), (16, 8, 20, 2.0), (9, 1, 3, 1.0),
             (40, 4, 0, 1.0), (130, 4, 1, 1.0), (25, 5, 50, 3.0), (12, 7, 10, 1.0)]
    for ci, (B, n, iters, scale) in enumerate(cases):
        g = torch.Generator().manual_seed(5000 + ci)
        H = scale * torch.randn(B, n, n, generator=g) + 2.0 * torch.eye(n)
        G = torch.randn(B, n, n, generator=g)
        Hr = H.clone().requires_grad_(True)
        P = MHC._sinkhorn_knopp(SimpleNamespace(sinkhorn_iters=iters), Hr)
        P.backward(G)
        key = f"c{ci}"
        rec[f"{key}_meta"] = np.array([B, n, iters])
        for name, t in (("H", H), ("G", G), ("P", P.detach()), ("dH", Hr.grad)):
            rec[f"{key}_{name}"] = t.numpy()
    np.savez_compressed(os.path.join(out, "sinkhorn.npz"), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HC_REFERENCE"),
                    help="root of a pjjajal/hyperconnections checkout (default: $HC_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", nargs="*", help="generate only these fixture groups (function names without gen_)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set HC_REFERENCE to the reference checkout")
    ref_expm, ref_small = _import_reference(args.reference)
    groups = {
        "expm": lambda: gen_expm(ref_expm, args.out),
        "stream_mix": lambda: gen_stream_mix(ref_small, args.out),
        "stream_mix_large_n": lambda: gen_stream_mix_large_n(ref_small, args.out),
        "fused": lambda: gen_fused(ref_small, args.out),
        "rw": lambda: gen_rw(ref_small, args.out),
        "layer": lambda: gen_layer(args.reference, args.out),
        "module": lambda: gen_module(args.out),
        "module_ghc_mhc": lambda: gen_module_ghc_mhc(args.out),
        "sinkhorn": lambda: gen_sinkhorn(args.out),
        "generator": lambda: gen_generator(args.out),
    }
    for name in args.only or groups:
        groups[name]()
    for name in sorted(os.listdir(args.out)):
        if name.endswith(".npz"):
            print(name, os.path.getsize(os.path.join(args.out, name)), "bytes")


if __name__ == "__main__":
    main()
