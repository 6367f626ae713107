"""CPU oracle of PageLoRA's decode hot path -- TEST INFRASTRUCTURE ONLY.

Plain numpy / Python restatements of the reference algorithms, each
function citing the reference file:line it follows.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this package, and only as the checker or the timed CPU baseline;
the product (``pagelora_b200``) never calls into it.

Pinning: the restatements are checked against golden vectors produced by
running the reference's own code in the build container
(``tests/golden/make_golden.py``) and against the known answers of the
reference's test-suite (page-table goldens, finite-mask attention case).
"""
