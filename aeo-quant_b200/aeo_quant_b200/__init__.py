"""aeo_quant_b200 — B200 (sm_100a) kernels behind aeo_quant's quantized MoE expert API.

Drop-in modules mirroring the reference package layout:

* ``aeo_quant_b200.gpu.quant``         <- ``aeo_quant.gpu.quant``
* ``aeo_quant_b200.gpu.nvfp4_matmul``  <- ``aeo_quant.gpu.nvfp4_matmul``
* ``aeo_quant_b200.bridges.gemma4``    <- ``aeo_quant.bridges.gemma4`` (expert class swap)

Every op runs hand-written CUDA through the C ABI in ``include/aeoq.h``.
"""
from ._capi import AeoqError, lib_path, load  # noqa: F401

__version__ = "0.1.0"
