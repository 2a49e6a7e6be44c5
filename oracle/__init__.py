"""CPU oracle for futudiffu_b200 -- TEST INFRASTRUCTURE ONLY.

A plain restatement, in torch CPU / numpy, of the arithmetic of the reference
(sqcu/futudiffu) for the quantized DiT hot path.  Every function cites the
reference file:line it follows.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s CPU baseline
leg; the product path (``futudiffu_b200``) never calls it and has no CPU
fallback.

Pinning: ``tests/golden/`` holds fixtures produced by running the reference's
own CPU-runnable code in this repository's build container
(``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py`` checks this
oracle against them.  Kernel-only arithmetic that the reference exposes only as
Triton GPU code (the attention kernels' online softmax, the blockwise GEMM's
promotion order) is restated from the reference source and pinned through
shared sub-steps (quantisers, smoothing, dequantisation) plus the
reference's own cosine thresholds.
"""
