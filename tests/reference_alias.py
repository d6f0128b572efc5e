"""Point the reference's ``hyperconnections.ops`` at ``hyperconnections_b200.ops``.

Importing this module (as a pytest plugin with ``-p tests.reference_alias``,
or before running one of the reference's scripts) imports the reference
package from baseline/_ref with ``hyperconnections.ops``,
``hyperconnections.ops.stream_mix`` and ``hyperconnections.ops.expm``
resolving to this package's operators, so every ``from hyperconnections.ops
import ...`` in the reference binds the B200 kernels. It prints one line to
stderr naming the module the reference's ``stream_mix_add`` now comes from.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import hyperconnections_b200.ops as _b200_ops  # noqa: E402
from baseline import reference_env  # noqa: E402

_ref = reference_env.import_reference(ops=_b200_ops)
_bound = sys.modules["hyperconnections.ops.stream_mix"].stream_mix_add
assert _bound is _b200_ops.stream_mix_add
print(f"reference_alias: hyperconnections.ops.stream_mix_add -> {_bound.__module__}", file=sys.stderr, flush=True)
