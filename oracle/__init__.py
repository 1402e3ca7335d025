"""CPU oracle for the PseudoBrain hot path. TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms of defnotean/pseudobrain's
data-parallel hot path:

* ``oracle.gdn``   -- the gated delta rule: the per-step recurrence
  (pseudobrain/gated_deltanet.py:93-107) and the chunkwise WY algorithm
  (pseudobrain/gated_deltanet.py:110-165).
* ``oracle.quest`` -- Quest page-bounded exact memory: page bounds
  (pseudobrain/exact_memory.py:43-50), archive append (:66-85), flat bound score,
  top-k page selection and gather (:88-152), and the exact attention over
  retrieved pages plus the sliding window (pseudobrain/transplant.py:612-628); and the
  canonical-order page scores (fp32, dimension order) that pin the kernels' page
  selections bit for bit.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline and
reference legs may import it, and only as the checker or as the timed CPU
baseline. The product (``pseudobrain_b200``) never imports it: it has no CPU
fallback and fails loudly when its CUDA library is missing.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
PyTorch functions on seeded inputs and stored their outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against
them.
"""
