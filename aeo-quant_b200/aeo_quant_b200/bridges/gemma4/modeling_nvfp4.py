"""Gemma4TextExpertsNVFP4 on B200 — drop-in for
``aeo_quant.bridges.gemma4.modeling_nvfp4``.

Same class name, base class, buffer names/shapes/dtypes and forward
signature as aeo_quant ``src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:46-255``,
so ``from_pretrained`` under the class swap loads the same NVFP4 checkpoint.

* One token (``hidden_states.shape[0] == 1``): the whole
  ``_forward_decode_3d`` (:132-186) is ``aeoq_moe_nvfp4_decode`` — two
  kernel launches, no host sync, capturable in a CUDA graph.
* More tokens: ``_forward_prefill`` (:188-255) semantics — one global
  activation quant, per-expert gate_up GEMM, GeGLU, per-expert re-quantized
  down GEMM, weighted bf16 combine in ascending expert order.
"""
from __future__ import annotations

import os
from contextlib import nullcontext

import torch
import torch.nn as nn
from transformers.activations import ACT2FN
from transformers.models.gemma4.modeling_gemma4 import Gemma4TextExperts

from ... import _capi as A
from ...gpu.quant import NVFP4_BLOCK_SIZE
from . import moe_ops

_MOE_TRACE = os.environ.get("AEO_MOE_TRACE") == "1"


def _moe_range(name: str):
    if _MOE_TRACE:
        return torch.cuda.nvtx.range(name)
    return nullcontext()


class Gemma4TextExpertsNVFP4(Gemma4TextExperts):
    """NVFP4 expert container + B200 forward (modeling_nvfp4.py:46-130)."""

    gate_up_proj: torch.Tensor
    gate_up_proj_scale: torch.Tensor
    gate_up_proj_scale_2: torch.Tensor
    down_proj: torch.Tensor
    down_proj_scale: torch.Tensor
    down_proj_scale_2: torch.Tensor
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

        ne = self.num_experts
        im = self.intermediate_dim
        hd = self.hidden_dim
        bs = NVFP4_BLOCK_SIZE
        self.register_buffer("gate_up_proj", torch.empty(ne, 2 * im, hd // 2, dtype=torch.uint8),
                             persistent=True)
        self.register_buffer("down_proj", torch.empty(ne, hd, im // 2, dtype=torch.uint8),
                             persistent=True)
        self.register_buffer("gate_up_proj_scale",
                             torch.empty(ne, 2 * im, hd // bs, dtype=torch.float8_e4m3fn), persistent=True)
        self.register_buffer("down_proj_scale",
                             torch.empty(ne, hd, im // bs, dtype=torch.float8_e4m3fn), persistent=True)
        self.register_buffer("gate_up_proj_scale_2", torch.tensor(0.0, dtype=torch.float32), persistent=True)
        self.register_buffer("down_proj_scale_2", torch.tensor(0.0, dtype=torch.float32), persistent=True)

    def forward(self, hidden_states, top_k_index, top_k_weights):
        """Shape dispatch of the reference (modeling_nvfp4.py:114-130)."""
        if hidden_states.shape[0] == 1:
            return self._forward_decode_3d(hidden_states, top_k_index, top_k_weights)
        return self._forward_prefill(hidden_states, top_k_index, top_k_weights)

    def _decode_launcher(self):
        """The cached one-token launcher, rebuilt when a weight buffer moves
        or is modified in place."""
        bufs = (self.gate_up_proj, self.gate_up_proj_scale, self.gate_up_proj_scale_2,
                self.down_proj, self.down_proj_scale, self.down_proj_scale_2)
        key = tuple((b.data_ptr(), b._version) for b in bufs)
        cached = self.__dict__.get("_decode_cache")
        if cached is None or cached[0] != key:
            cached = (key, moe_ops.DecodeLauncher(*bufs))
            self.__dict__["_decode_cache"] = cached
        return cached[1]

    def _forward_decode_3d(self, hidden_states, top_k_index, top_k_weights):
        """One token: fused gather GEMV pair (modeling_nvfp4.py:132-186)."""
        if not hidden_states.is_cuda:
            raise moe_ops.A.AeoqError("aeo_quant_b200 runs on CUDA tensors only (no CPU path); "
                                      f"got a tensor on {hidden_states.device}")
        with _moe_range("nvfp4_moe_decode_fused"):
            out = self._decode_launcher()(hidden_states, top_k_index, top_k_weights)
        return out if out.dtype == hidden_states.dtype else out.to(hidden_states.dtype)

    def _forward_prefill(self, hidden_states, top_k_index, top_k_weights):
        """Many tokens (modeling_nvfp4.py:188-255)."""
        with _moe_range("nvfp4_moe_prefill"):
            return moe_ops.nvfp4_prefill(
                hidden_states, top_k_index, top_k_weights,
                self.gate_up_proj, self.gate_up_proj_scale, self.gate_up_proj_scale_2,
                self.down_proj, self.down_proj_scale, self.down_proj_scale_2,
                self.num_experts)
