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


def _from_pretrained(model_id_or_path, kwargs):
    """``AutoModelForCausalLM.from_pretrained`` with the reference's
    defaults (bf16, ``device_map="cuda"``, loader.py:87-88, :125-126).
    ``device_map`` needs the ``accelerate`` package; without it, a
    single-device map (a string or ``torch.device``) is honoured by loading
    on the host and moving the model, and any other map is an error."""
    from transformers import AutoModelForCausalLM
    kwargs.setdefault("dtype", torch.bfloat16)
    kwargs.setdefault("device_map", "cuda")
    dev = kwargs.get("device_map")
    move_to = None
    if dev is not None:
        try:
            import accelerate  # noqa: F401
        except ImportError:
            if not isinstance(dev, (str, torch.device)) or str(dev) == "auto":
                raise ValueError(f"device_map={dev!r} needs the accelerate package; pass a single device") from None
            kwargs.pop("device_map")
            move_to = torch.device(dev)
    model = AutoModelForCausalLM.from_pretrained(model_id_or_path, **kwargs)
    if move_to is not None:
        model = model.to(move_to)
    return model


def _install_fused_routers(model):
    """Fused router forward on a model whose weights are on a GPU, for every
    router whose shapes the kernel takes (the others keep HF's forward)."""
    p = next(model.parameters(), None)
    if p is not None and p.is_cuda:
        swap_routers(model, only_supported=True)
    return model


def load_gemma4(model_id_or_path, *, quant_format="fp8", **from_pretrained_kwargs):
    """Dispatch by format (loader.py:67-76)."""
    if quant_format == "nvfp4":
        return load_gemma4_nvfp4(model_id_or_path, **from_pretrained_kwargs)
    return load_gemma4_fp8(model_id_or_path, **from_pretrained_kwargs)


def load_gemma4_fp8(model_id_or_path, **from_pretrained_kwargs):
    """Load an FP8 checkpoint under the class swap (loader.py:79-92). On a
    GPU the routers get the fused forward as well."""
    with gemma4_experts_fp8_class_swap():
        model = _from_pretrained(model_id_or_path, from_pretrained_kwargs)
    _preconvert_fp8_scales(model)
    return _install_fused_routers(model)


def load_gemma4_nvfp4(model_id_or_path, **from_pretrained_kwargs):
    """Load an NVFP4 checkpoint (``checkpoint.build_checkpoint_nvfp4``'s
    output, or the reference builder's) under the class swap
    (loader.py:111-138). The 0-d bf16 ``*_scale_2`` tensors load into the
    modules' fp32 buffers. On a GPU the routers get the fused forward as
    well."""
    with _gemma4_experts_nvfp4_class_swap():
        model = _from_pretrained(model_id_or_path, from_pretrained_kwargs)
    return _install_fused_routers(model)


@torch.no_grad()
def quantize_experts_to_nvfp4(model):
    """Replace every bf16 ``Gemma4TextExperts`` in ``model`` by a
    ``Gemma4TextExpertsNVFP4`` holding its NVFP4 quantization, on the
    experts' device.

    This is the expert step of the reference's checkpoint builder
    (``examples/build_checkpoint_nvfp4.py:133-151``): each fused 3-D expert
    tensor goes through ``quantize_3d_to_nvfp4`` and becomes ``<proj>``
    (packed E2M1), ``<proj>_scale`` (e4m3 block scales) and ``<proj>_scale_2``
    (the tensor scale, held as a 0-d fp32 buffer as after loading). Here it
    runs on the GPU kernels, one layer at a time, and each layer's bf16
    weights are released as soon as its NVFP4 copy exists. Returns the
    number of modules converted."""
    from ...gpu.quant import quantize_3d_to_nvfp4

    targets = []
    for name, mod in model.named_modules():
        for child_name, child in mod.named_children():
            if type(child) is modeling_gemma4.Gemma4TextExperts:
                targets.append((mod, child_name, child))
    for parent, child_name, old in targets:
        dev = old.gate_up_proj.device
        cfg = _ExpertShape(old)
        new = Gemma4TextExpertsNVFP4(cfg).to(dev)
        for proj in ("gate_up_proj", "down_proj"):
            packed, block_scale, tensor_scale = quantize_3d_to_nvfp4(getattr(old, proj).detach().to(torch.bfloat16))
            getattr(new, proj).copy_(packed)
            getattr(new, f"{proj}_scale").copy_(block_scale)
            getattr(new, f"{proj}_scale_2").copy_(tensor_scale.float())
            del packed, block_scale, tensor_scale
        setattr(parent, child_name, new)
        del old
    return len(targets)


class _ExpertShape:
    """The config fields ``Gemma4TextExpertsNVFP4.__init__`` reads, taken
    from an existing bf16 expert module."""

    def __init__(self, experts):
        E, two_i, H = experts.gate_up_proj.shape
        self.num_experts = E
        self.hidden_size = H
        self.moe_intermediate_size = two_i // 2
        self.hidden_activation = "gelu_pytorch_tanh"


def gemma4_router_class_swap():
    """Swap in ``Gemma4TextRouterB200`` for ``Gemma4TextRouter`` while a
    model is built (same parameters, fused forward)."""
    from .router import Gemma4TextRouterB200

    @contextlib.contextmanager
    def _cm():
        original = modeling_gemma4.Gemma4TextRouter
        modeling_gemma4.Gemma4TextRouter = Gemma4TextRouterB200
        try:
            yield
        finally:
            modeling_gemma4.Gemma4TextRouter = original
    return _cm()


def swap_routers(model, only_supported: bool = False):
    """Give every ``Gemma4TextRouter`` in a built model the fused forward
    (its parameters stay where they are). With ``only_supported``, routers
    whose shapes the kernel does not take are left as they are. Returns the
    number swapped."""
    from .router import Gemma4TextRouterB200, router_supported
    n = 0
    for mod in model.modules():
        if type(mod) is modeling_gemma4.Gemma4TextRouter and (not only_supported or router_supported(mod)):
            mod.__class__ = Gemma4TextRouterB200
            n += 1
    return n
