"""CPU oracle for the telescoping-attention hot path -- TEST INFRASTRUCTURE.

This package is a plain-numpy / pure-Python restatement of the reference
algorithm (Knarf04/telescope_cache ``reference.py`` and
``telescoping_attn/range_spec.py``).  It exists only to check the CUDA path:

* ``tests/`` compare the CUDA kernels against it on seeded inputs;
* ``__graft_entry__.smoke()`` checks one small CUDA call against it;
* ``bench.py`` times it as the CPU baseline (``cpu_baseline`` /
  ``--impl reference``).

Nothing in ``telescope_cache_b200`` imports it: the product path has no CPU
fallback and fails loudly when its CUDA library is missing.

The oracle is pinned against golden vectors produced by running the
reference itself (``tests/golden/make_golden.py``; checked by
``tests/test_oracle_golden.py``).

Modules
-------
schedule   integer schedule: activation times, per-query level ranges (the
           analytic ruler/slot formulation), hulls, coarsest span, decode
           ring capacities, chronological bin distances
numerics   float64 restatement of the builder, forward, backward, post-ops
           and incremental decode, by per-query visible-entry enumeration
"""
