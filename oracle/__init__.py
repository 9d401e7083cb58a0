"""CPU oracle for the quantized MoE expert path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of aeo_quant's quantized
expert path (quantizers in ``src/aeo_quant/gpu/quant.py``, the block-scaled
GEMM contract of ``src/aeo_quant/gpu/nvfp4_matmul.py``, the FP8 rowwise
``_scaled_mm`` contract and the expert forwards in
``src/aeo_quant/bridges/gemma4/``). It is the checker the CUDA library is
compared against, and nothing else:

* only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
  ``bench.py`` import it;
* the product package (``aeo-quant_b200/aeo_quant_b200``) never imports it
  and has no CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own
Python quantizers and expert forwards in the build container and commits
their outputs as fixtures; ``tests/test_oracle_golden.py`` checks this
package against them. The GEMM arithmetic itself lives in third-party code
(Triton ``tl.dot_scaled``, cuBLASLt ``_scaled_mm``); for those the fixtures
hold the reference forwards with the GEMM call restated, so the GEMM
contract is pinned by its published definition, not by reference outputs.
"""
from . import gemm, moe, numerics, quant, router  # noqa: F401
