"""CPU oracle for the slice/deslice coupling -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithm of the reference
implementation (Shizheng-Wen/flashslice v0.3.0) for the path that
``flashslice_b200`` accelerates: ``fused_slice`` / ``fused_deslice``, their
recompute-based backward and the per-point softmax statistics.

* ``oracle.coupling`` -- numpy, any float dtype (fp64 is the truth): the
  forward of both ops, their analytic backward and the statistics (m, l).
* ``oracle.eager_torch`` -- the reference's own eager op math
  (``bench/parity_ops.py:59-79``) restated with torch CPU tensors and
  autograd; in fp32 it is "the reference's own implementation" that the
  tolerances are quoted against, and it is the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference``) may import this package, and
only as the checker or the timed CPU baseline. The product path
(``flashslice_b200``) never imports it and has no CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` generated the fixtures in
``tests/golden/`` by importing the reference in the build container (its
eager math in fp64 with autograd, and its Triton kernels under
``TRITON_INTERPRET=1`` for the statistics); ``tests/test_oracle_golden.py``
holds this oracle to them.
"""
