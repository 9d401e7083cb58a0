"""Gemma4TextExpertsFP8 on B200 — drop-in for ``aeo_quant.bridges.gemma4.modeling``.

Same class name, base class, parameter/buffer names, shapes and dtypes and
forward signature as aeo_quant ``src/aeo_quant/bridges/gemma4/modeling.py:29-146``,
so ``from_pretrained`` under the FP8 class swap loads the same checkpoint:
``gate_up_proj`` (E, 2I, H) and ``down_proj`` (E, H, I) float8_e4m3fn
Parameters, ``gate_up_proj_scale`` (E, 2I, 1) and ``down_proj_scale``
(E, H, 1) bf16 buffers (preconverted to (E, 1, N) f32 by the loader).

The forward keeps the reference's numerics (per-row dynamic e4m3 input
quantization, bf16((acc * sa) * sb) GEMMs, bf16 GeGLU, bf16 weighting and
the bf16 ``index_add_`` fold in ascending expert order) and runs as six
device launches without host synchronisation: routing, gathered row
quantization, grouped gate_up GEMM with the GeGLU epilogue, row
re-quantization, grouped down GEMM with the weighting epilogue, combine.
"""
from __future__ import annotations

import os
from contextlib import nullcontext

import torch
import torch.nn as nn
from transformers.activations import ACT2FN
from transformers.models.gemma4.modeling_gemma4 import Gemma4TextExperts

from . import moe_ops

_MOE_TRACE = os.environ.get("AEO_MOE_TRACE") == "1"


def _moe_range(name: str):
    if _MOE_TRACE:
        return torch.cuda.nvtx.range(name)
    return nullcontext()


class Gemma4TextExpertsFP8(Gemma4TextExperts):
    """FP8 expert container + B200 forward (modeling.py:29-146)."""

    gate_up_proj: torch.Tensor
    gate_up_proj_scale: torch.Tensor
    down_proj: torch.Tensor
    down_proj_scale: torch.Tensor
    num_experts: int

    def __init__(self, config):
        nn.Module.__init__(self)
        self.num_experts = config.num_experts
        self.hidden_dim = config.hidden_size
        self.intermediate_dim = config.moe_intermediate_size
        self.act_fn = ACT2FN[config.hidden_activation]
        act = getattr(config, "hidden_activation", "gelu_pytorch_tanh")
        if act not in ("gelu_pytorch_tanh", "gelu_tanh"):
            raise ValueError(f"hidden_activation={act!r} is not supported by the fused kernels "
                             "(gelu_pytorch_tanh only)")
        ne, im, hd = self.num_experts, self.intermediate_dim, self.hidden_dim
        self.gate_up_proj = nn.Parameter(torch.empty(ne, 2 * im, hd, dtype=torch.float8_e4m3fn),
                                         requires_grad=False)
        self.down_proj = nn.Parameter(torch.empty(ne, hd, im, dtype=torch.float8_e4m3fn), requires_grad=False)
        self.register_buffer("gate_up_proj_scale", torch.empty(ne, 2 * im, 1, dtype=torch.bfloat16),
                             persistent=True)
        self.register_buffer("down_proj_scale", torch.empty(ne, hd, 1, dtype=torch.bfloat16), persistent=True)
        self._sb_cache: dict = {}

    @staticmethod
    def _fp8_linear(x_bf16, w_fp8, scale_w_1xN):
        """FP8 matmul with per-row dynamic input quantization (modeling.py:89-108)."""
        return moe_ops.fp8_linear(x_bf16, w_fp8, scale_w_1xN)

    def _scales(self, name: str, N: int) -> torch.Tensor:
        buf = getattr(self, name)
        key = (name, buf.data_ptr(), tuple(buf.shape), buf.dtype, buf._version)
        hit = self._sb_cache.get(name)
        if hit is not None and hit[0] == key:
            return hit[1]
        sb = moe_ops.fp8_scale_rows(buf, self.num_experts, N)
        self._sb_cache[name] = (key, sb)
        return sb

    def forward(self, hidden_states, top_k_index, top_k_weights):
        if hidden_states.dtype != torch.bfloat16:
            raise ValueError(f"hidden_states must be bfloat16, got {hidden_states.dtype}")
        E, H, I = self.num_experts, self.hidden_dim, self.intermediate_dim
        with _moe_range("fp8_moe"), torch.no_grad():
            return moe_ops.fp8_experts_grouped(
                hidden_states, top_k_index, top_k_weights, self.gate_up_proj, self._scales("gate_up_proj_scale", 2 * I),
                self.down_proj, self._scales("down_proj_scale", H))
