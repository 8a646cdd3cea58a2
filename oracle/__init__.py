"""CPU oracle for the HCLSM hot path — TEST INFRASTRUCTURE ONLY.

Restatements of the reference algorithms (RightNow-AI/hclsm) used as the parity
checker and as the timed CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg import this package; the product path
(``hclsm_b200``) never does.

Pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).
"""
