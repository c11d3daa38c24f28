"""CPU oracle for the FSCTEP message-passing hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the reference algorithm of
Parity-LRX/FSCTEP (``molecular_force_field``) for the per-edge Cartesian
tensor-product layers and their force/virial backward.  Every function cites
the reference file:line it follows (paths relative to the reference project).

Rules that apply to everything in here:

* Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
  leg (``--impl reference`` and the ``cpu_baseline`` key) may import it, and
  only as the checker or the timed CPU baseline.  The product path
  (``fsctep_b200``) never imports, calls or links anything under ``oracle/``.
* The oracle is pinned against golden vectors produced by the reference itself
  (``tests/golden/make_golden.py`` imports the unmodified reference with three
  import shims and records its outputs); ``tests/test_oracle_golden.py`` checks
  the restatement against them.
* The radial basis comes from a third-party package absent from the reference
  tree (``e3nn.math.soft_one_hot_linspace``, pinned ``e3nn>=0.4.4,<0.6.0`` in
  the reference ``setup.py:81``).  ``oracle/radial.py`` restates its published
  formula; the golden generator uses that same restatement as its shim, so
  parity at that one boundary is conditional on the restatement ("parity
  unpinned" for the radial basis alone; everything downstream of it is pinned).
"""
