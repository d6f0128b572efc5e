"""Install the reference (pjjajal/hyperconnections) into baseline/_ref.

    python baseline/install_reference.py --reference <checkout>   (or $HC_REFERENCE)

baseline/_ref is git-ignored; it travels with the working tree to GPU hosts,
where the checkout itself is absent. It serves bench.py's reference arm and
CPU baseline (the reference's own eager CPU path) and the drop-in tests that
run the reference's own callers of the ops on this package's kernels.

Steps:
1. the offline install of the contract: ``pip install --no-index
   --no-build-isolation --find-links /opt/wheelhouse --target baseline/_ref
   <checkout>``;
2. when pip cannot build the project (its build backend, hatchling, is not in
   the offline wheelhouse), the ``hyperconnections`` package directory is
   copied unmodified: for this pure-Python project that is exactly what its
   wheel would install;
3. the reference's own callers of the ops, ``tests/test_ops.py``,
   ``tests/conftest.py`` and ``benchmarks/stream_mix_bench.py``, are copied
   unmodified into baseline/_ref/_callers/.
baseline/_ref/INSTALL.txt records what happened.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
CALLERS = ("tests/test_ops.py", "tests/conftest.py", "benchmarks/stream_mix_bench.py")


def install(reference: str, force: bool = False) -> str:
    """Install (or keep) baseline/_ref; returns a one-line outcome."""
    pkg = os.path.join(TARGET, "hyperconnections")
    if os.path.isdir(pkg) and not force:
        return "already installed"
    if os.path.isdir(TARGET):
        shutil.rmtree(TARGET)
    os.makedirs(TARGET)
    cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", TARGET, reference]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode == 0 and os.path.isdir(pkg):
        outcome = "pip install --target: ok"
    else:
        last = (proc.stderr or proc.stdout).strip().splitlines()
        why = last[-1] if last else f"rc {proc.returncode}"
        shutil.rmtree(TARGET)
        os.makedirs(TARGET)
        shutil.copytree(os.path.join(reference, "hyperconnections"), pkg,
                        ignore=shutil.ignore_patterns("__pycache__"))
        outcome = f"pip install failed ({why}); package directory copied unmodified"
    callers = os.path.join(TARGET, "_callers")
    for rel in CALLERS:
        src = os.path.join(reference, rel)
        dst = os.path.join(callers, rel)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        shutil.copy2(src, dst)
    with open(os.path.join(TARGET, "INSTALL.txt"), "w") as fh:
        fh.write(outcome + "\n")
        fh.write("callers: " + ", ".join(CALLERS) + "\n")
    return outcome


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", default=os.environ.get("HC_REFERENCE"),
                    help="root of a pjjajal/hyperconnections checkout (default: $HC_REFERENCE)")
    ap.add_argument("--force", action="store_true", help="reinstall even if baseline/_ref exists")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference or set HC_REFERENCE to the reference checkout")
    print(install(args.reference, args.force))


if __name__ == "__main__":
    main()
