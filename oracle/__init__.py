"""CPU oracle for the compressed-cache attention path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy and plain Python, the reference algorithms that
libabkv.so implements on the GPU.  Each function cites the reference file:line
it follows (paths are relative to the AbridgeKV project root).  It is imported
only by tests/, by __graft_entry__.smoke() as the checker, and by bench.py's
CPU-baseline leg / reference arm.  The product path (abridgekv_b200) never
imports it and has no CPU fallback.

Pinning: tests/golden/ holds outputs of the reference's own code (imported
from the AbridgeKV sources in the build container by tests/golden/make_golden.py)
and every restatement here is checked against them by tests/test_oracle_golden.py.
"""
