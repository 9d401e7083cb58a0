"""Class-swap loaders — drop-in for ``aeo_quant.bridges.gemma4.loader``.

Same context managers and loaders as aeo_quant
``src/aeo_quant/bridges/gemma4/loader.py:32-138``: during ``from_pretrained``
``transformers...modeling_gemma4.Gemma4TextExperts`` is replaced by the B200
subclass and restored in ``finally``.
"""
from __future__ import annotations

import contextlib

import torch
from transformers.models.gemma4 import modeling_gemma4

from .modeling_nvfp4 import Gemma4TextExpertsNVFP4


@contextlib.contextmanager
def _swap(cls):
    original = modeling_gemma4.Gemma4TextExperts
    modeling_gemma4.Gemma4TextExperts = cls
    try:
        yield
    finally:
        modeling_gemma4.Gemma4TextExperts = original


def gemma4_experts_fp8_class_swap():
    """Swap in ``Gemma4TextExpertsFP8`` (loader.py:32-44)."""
    from .modeling import Gemma4TextExpertsFP8
    return _swap(Gemma4TextExpertsFP8)


def _gemma4_experts_nvfp4_class_swap():
    """Swap in ``Gemma4TextExpertsNVFP4`` (loader.py:100-108)."""
    return _swap(Gemma4TextExpertsNVFP4)


def _preconvert_fp8_scales(model):
    """(E, N, 1) bf16 scales -> (E, 1, N) fp32, in place (loader.py:47-64)."""
    from .modeling import Gemma4TextExpertsFP8
    for module in model.modules():
        if isinstance(module, Gemma4TextExpertsFP8):
            module.gate_up_proj_scale = module.gate_up_proj_scale.squeeze(-1).unsqueeze(1).float().contiguous()
            module.down_proj_scale = module.down_proj_scale.squeeze(-1).unsqueeze(1).float().contiguous()


def load_gemma4(model_id_or_path, *, quant_format="fp8", **from_pretrained_kwargs):
    """Dispatch by format (loader.py:67-76)."""
    if quant_format == "nvfp4":
        return load_gemma4_nvfp4(model_id_or_path, **from_pretrained_kwargs)
    return load_gemma4_fp8(model_id_or_path, **from_pretrained_kwargs)


def load_gemma4_fp8(model_id_or_path, **from_pretrained_kwargs):
    """Load an FP8 checkpoint under the class swap (loader.py:79-92)."""
    from transformers import AutoModelForCausalLM
    from_pretrained_kwargs.setdefault("dtype", torch.bfloat16)
    from_pretrained_kwargs.setdefault("device_map", "cuda")
    with gemma4_experts_fp8_class_swap():
        model = AutoModelForCausalLM.from_pretrained(model_id_or_path, **from_pretrained_kwargs)
    _preconvert_fp8_scales(model)
    return model


def load_gemma4_nvfp4(model_id_or_path, **from_pretrained_kwargs):
    """Load an NVFP4 checkpoint under the class swap (loader.py:111-138)."""
    from transformers import AutoModelForCausalLM
    from_pretrained_kwargs.setdefault("dtype", torch.bfloat16)
    from_pretrained_kwargs.setdefault("device_map", "cuda")
    with _gemma4_experts_nvfp4_class_swap():
        model = AutoModelForCausalLM.from_pretrained(model_id_or_path, **from_pretrained_kwargs)
    return model
