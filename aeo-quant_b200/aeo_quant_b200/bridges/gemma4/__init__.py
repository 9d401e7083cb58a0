"""Gemma 4 expert class swap (drop-in for ``aeo_quant.bridges.gemma4``)."""
from .loader import (gemma4_experts_fp8_class_swap, load_gemma4, load_gemma4_fp8,  # noqa: F401
                     load_gemma4_nvfp4)
from .modeling import Gemma4TextExpertsFP8  # noqa: F401
from .modeling_nvfp4 import Gemma4TextExpertsNVFP4  # noqa: F401
