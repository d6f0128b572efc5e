"""Import the reference (pjjajal/hyperconnections) installed in baseline/_ref.

BASELINE AND TEST INFRASTRUCTURE: bench.py's reference arm and CPU baseline
and the drop-in tests use it; the product package never imports it.

The reference imports ``timm.models.layers.trunc_normal_`` (cghc.py:9,
mhc.py:7), and timm is not installed here: when ``import timm`` fails, a
stand-in module exposing torch's own ``torch.nn.init.trunc_normal_`` under
that name is registered first (the reference only calls it at init). Nothing
of the reference is modified.

``import_reference(ops=...)`` can make ``hyperconnections.ops`` and its
``stream_mix`` / ``expm`` submodules resolve to another module, this
package's ``hyperconnections_b200.ops``: every ``from hyperconnections.ops
import ...`` in the reference (cghc.py:11, benchmarks/stream_mix_bench.py:35,
tests/test_ops.py:17) then binds this package's functions.
"""

from __future__ import annotations

import importlib
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
CALLERS_DIR = os.path.join(REF_DIR, "_callers")


def available() -> bool:
    """True when baseline/_ref holds the reference package."""
    return os.path.isfile(os.path.join(REF_DIR, "hyperconnections", "cghc.py"))


def _timm_stand_in() -> None:
    try:
        import timm.models.layers  # noqa: F401
        return
    except Exception:
        pass
    import torch

    timm = types.ModuleType("timm")
    models = types.ModuleType("timm.models")
    layers = types.ModuleType("timm.models.layers")
    layers.trunc_normal_ = torch.nn.init.trunc_normal_
    timm.models, models.layers = models, layers
    sys.modules.update({"timm": timm, "timm.models": models, "timm.models.layers": layers})


def _forget_reference() -> None:
    for name in [k for k in sys.modules if k == "hyperconnections" or k.startswith("hyperconnections.")]:
        del sys.modules[name]


def import_reference(ops=None):
    """Import the reference package from baseline/_ref (a fresh import every
    call). With ``ops`` (a module with ``stream_mix`` and ``expm``
    submodules), ``hyperconnections.ops`` resolves to it."""
    if not available():
        raise RuntimeError(f"the reference is not installed in {REF_DIR} (baseline/install_reference.py)")
    _timm_stand_in()
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    _forget_reference()
    if ops is not None:
        sys.modules["hyperconnections.ops"] = ops
        sys.modules["hyperconnections.ops.stream_mix"] = ops.stream_mix
        sys.modules["hyperconnections.ops.expm"] = ops.expm
    return importlib.import_module("hyperconnections")


def import_reference_ops():
    """The reference's own ``hyperconnections.ops`` (expm_t18, stream_mix_add)."""
    import_reference()
    return importlib.import_module("hyperconnections.ops")


def caller_path(rel: str) -> str:
    """Path of one of the reference's own callers copied at install time
    (tests/test_ops.py, tests/conftest.py, benchmarks/stream_mix_bench.py)."""
    return os.path.join(CALLERS_DIR, rel)
