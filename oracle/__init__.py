"""CPU oracle for the softhier-ops hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference's host-side algorithms for the operator
library path: the 32-bit LCG test-data generator (softhier_mlir/testing/lcg.py), the per-op
numpy references of tests/gvsoc/run.py (152-158, 921-934), and the SigLIP encoder-layer
reference (softhier_mlir/testing/siglip_ref.py:9-45). It is the checker the parity tests,
`__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py` compare against.

Nothing in the product path (the CUDA library, its ctypes binding, the emitter or the
encoder driver) may import or call this package.

Pinning: the restatement is checked against golden vectors produced by the reference's own
Python modules (tests/golden/make_golden.py imports them from the reference checkout and
writes tests/golden/*.npz); tests/test_oracle.py compares the two.
"""
