"""CPU oracle for the Evoformer hot path: TEST INFRASTRUCTURE, not product code.

A float32/float64 PyTorch-CPU restatement of the fp32 ``ref_*`` functions and custom-VJP
formulas of mirditalab/colabfold-kernels v0.9.0 (each function cites the reference file:line
it follows).  Only the tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it; the product package never does and
fails loudly when its CUDA library is missing.

Pinning: the reference holds no golden vectors and needs JAX, which is not installed where
this was built.  ``tests/golden/make_golden.py`` therefore executes the reference's own
``ref_*`` source under a NumPy stand-in for ``jax.numpy`` and commits the outputs as
fixtures; ``tests/test_oracle_golden.py`` checks this restatement against them.  The deep-MSA
outer-product-mean and the Evoformer block wiring are not in the reference (they live in
ColabFold/AlphaFold): for those two compositions parity is unpinned.
"""
from oracle.reference_math import *  # noqa: F401,F403
