"""TEST INFRASTRUCTURE ONLY: the CPU checker for the int8 quantized-linear path.

Two checkers live here, neither of which the product ever imports:

* ``kz_oracle.c`` (loaded through :mod:`oracle.cpu`) restates the reference's
  quantize / dequantize / qlinear arithmetic in C and adds the W8A8 extensions
  (per-channel and per-row scales, int8 GEMM, fused epilogue).
* ``_ref/`` holds the reference's own C++ core compiled from its sources and
  re-bound with pybind11 (``ref_core_py.cpp``); :mod:`oracle.refpkg` imports the
  reference's unmodified Python package over it, where the reference checkout
  is present.

Parity is pinned: ``tests/test_oracle_golden.py`` checks ``kz_oracle.c`` against
golden vectors that ``tests/golden/gen_golden.py`` produced from the reference's
own Python running over the reference's own C++ core.
"""
