"""CPU oracle for the hyper-connections hot path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, what the
reference (pjjajal/hyperconnections) computes on its hot path, so that the
CUDA kernels can be checked against it:

* ``oracle.expm``       — expm_t18 (hyperconnections/ops/expm.py:65-106), its
                          autograd gradient, and the Pade [7/7] exponential;
* ``oracle.stream_mix`` — stream_mix_add forward/backward
                          (ops/stream_mix_small_nb.py:75-391) and the fused
                          read + mix + write step (cghc.py:410, :417, :449);
* ``oracle.torch_ref``  — the reference's eager PyTorch CPU path for the same
                          work (the timed CPU baseline).

Parity is pinned: tests/test_oracle_golden.py checks these functions against
fixtures produced by running the reference's own code
(tests/golden/make_golden.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker or the CPU baseline. The product package
``hyperconnections_b200`` never imports it.
"""
