"""CPU tests of the ring geometry (hc_debug_ring_geometry: the host
arithmetic every pipelined launch runs, no GPU needed): over every op, n, m,
block size and stream dtype the kernels take, the stages, consumer warps and
shared memory stay within what a B200 CTA can hold, and the shapes measured
for the side rows (the backward's one-row tensors fetched by the consumer
warps) take them."""

import ctypes

import pytest

from hyperconnections_b200 import _lib

FIELDS = ("ring", "stages", "consumers", "producers", "tpi", "sl", "ns", "stage_bytes", "smem_bytes", "side",
          "gram_mma", "grid")
SMEM_LIMIT = 232448          # shared memory of one B200 CTA (227 KB), static and dynamic together
SIDE_BUDGET = 220 * 1024     # stages + slots of a side-row ring (kSideSmemBudget)
TOKENS = 16384
BLOCKS = (64, 128, 384, 512, 640, 768, 1024, 1536, 2048, 4096)
DTYPES = {"bf16": _lib.HC_DTYPE_BF16, "f32": _lib.HC_DTYPE_F32}


@pytest.fixture(scope="module")
def lib():
    if not _lib.available():
        pytest.skip("libhcops.so is not built")
    return _lib.lib()


def geometry(lib, op, bwd, n, D, dtype="bf16", m=1, proj=False, T=TOKENS):
    out = (ctypes.c_int * len(FIELDS))()
    rc = lib.hc_debug_ring_geometry(op, int(bwd), n, m, int(proj), T, D, DTYPES[dtype], out, len(FIELDS))
    assert rc == 0, (op, bwd, n, m, D, dtype, rc)
    return dict(zip(FIELDS, out))


def cases():
    for dtype in DTYPES:
        for D in BLOCKS:
            for bwd in (0, 1):
                for n in range(1, 9):
                    yield (0, bwd, n, 1, False, D, dtype)
                    for proj in (False, True):
                        yield (1, bwd, n, 1, proj, D, dtype)
                for n in (9, 12, 16, 24, 32):  # stream_mix_add on the tensor-core ring (bf16 only)
                    yield (1, bwd, n, 1, False, D, dtype)
                for n, m in ((2, 1), (4, 1), (4, 2), (4, 4), (6, 3), (8, 4)):
                    yield (2, bwd, n, m, False, D, dtype)
                    for proj in (False, True):
                        yield (3, bwd, n, m, proj, D, dtype)


def test_every_ring_fits_a_cta(lib):
    rings = 0
    for op, bwd, n, m, proj, D, dtype in cases():
        g = geometry(lib, op, bwd, n, D, dtype, m, proj)
        if not g["ring"]:
            continue
        rings += 1
        what = (op, bwd, n, m, proj, D, dtype, g)
        assert 3 <= g["stages"] <= 32, what
        assert 1 <= g["consumers"] <= g["stages"] - 2, what
        assert 1 <= g["producers"] <= min(g["stages"], 32), what
        assert g["tpi"] >= 1 and (g["tpi"] == 1 or g["ns"] == 1), what
        assert g["sl"] * g["ns"] >= D and g["sl"] * (g["ns"] - 1) < D, what
        assert g["stages"] * g["stage_bytes"] <= g["smem_bytes"] <= SMEM_LIMIT - 1024, what
        assert g["grid"] == min(148, TOKENS), what
        if g["side"]:
            assert bwd and op in (0, 3) and g["ns"] == 1 and not g["gram_mma"], what
            assert g["smem_bytes"] <= SIDE_BUDGET, what
    assert rings > 500


def test_side_rows_where_measured(lib):
    g = geometry(lib, 0, 1, 4, 768)  # the headline backward
    assert (g["side"], g["stages"], g["consumers"], g["stage_bytes"], g["smem_bytes"]) == (1, 14, 8, 12288, 221184)
    assert geometry(lib, 0, 1, 2, 1024)["side"] == 1
    g = geometry(lib, 0, 1, 4, 1024)  # consumers trimmed for their slots
    assert g["side"] == 1 and g["consumers"] == 7 and g["stages"] >= 9
    assert geometry(lib, 0, 1, 3, 1024)["side"] == 0   # odd n: the plain ring measured faster
    assert geometry(lib, 0, 1, 4, 512)["side"] == 0    # items of two tokens: the plain ring
    assert geometry(lib, 0, 0, 4, 768)["side"] == 0    # forward
    assert geometry(lib, 3, 1, 4, 768, m=1)["side"] == 1
    assert geometry(lib, 3, 1, 4, 768, m=1, proj=True)["side"] == 0
    assert geometry(lib, 2, 1, 4, 768, m=1)["side"] == 0   # read backward
    assert geometry(lib, 1, 1, 4, 768)["side"] == 0        # stream_mix_add


def test_large_n_ring(lib):
    for n in (9, 16, 32):
        g = geometry(lib, 1, 1, n, 1536)
        assert g["ring"] and g["gram_mma"] == 2 and g["consumers"] == 7 and g["stages"] >= 9, (n, g)
        # stages and 1 KB of alignment slack within the tensor-core rings' 216 KB budget
        assert g["smem_bytes"] <= 216 * 1024 + 1024, (n, g)
    assert not geometry(lib, 1, 1, 16, 1536, dtype="f32")["ring"]  # fp32 streams take the CUDA-core kernels
    assert not geometry(lib, 1, 1, 16, 100)["ring"]                # D not a multiple of 64


def test_tuning_hook_reaches_the_side_rows(lib):
    try:
        assert lib.hc_debug_set_mix_tuning(0, 3, 1, 0) == 0
        g = geometry(lib, 0, 1, 4, 768)
        assert (g["side"], g["stages"], g["consumers"]) == (1, 3, 1)
    finally:
        assert lib.hc_debug_set_mix_tuning(0, 0, 0, 0) == 0


def test_rejects_bad_arguments(lib):
    out = (ctypes.c_int * len(FIELDS))()
    assert lib.hc_debug_ring_geometry(0, 1, 9, 1, 0, TOKENS, 768, _lib.HC_DTYPE_BF16, out, len(FIELDS)) != 0
    assert lib.hc_debug_ring_geometry(1, 1, 33, 1, 0, TOKENS, 768, _lib.HC_DTYPE_BF16, out, len(FIELDS)) != 0
    assert lib.hc_debug_ring_geometry(7, 1, 4, 1, 0, TOKENS, 768, _lib.HC_DTYPE_BF16, out, len(FIELDS)) != 0
    assert lib.hc_debug_ring_geometry(0, 1, 4, 1, 0, 0, 768, _lib.HC_DTYPE_BF16, out, len(FIELDS)) != 0
    assert lib.hc_debug_ring_geometry(0, 1, 4, 1, 0, TOKENS, 768, 9, out, len(FIELDS)) != 0
    assert lib.hc_debug_ring_geometry(0, 1, 4, 1, 0, TOKENS, 768, _lib.HC_DTYPE_BF16, None, 1) != 0
