"""LinearFP8 on B200: drop-in for ``aeo_quant.bridges.gemma4.linear_fp8``.

Same module (``weight`` (out, in) float8_e4m3fn Parameter, ``weight_scale``
(1, out) fp32 buffer, optional bf16 ``bias``), the same ``from_linear`` and
the same ``fp8_linear(x, w_fp8, scale_w, bias)`` function as aeo_quant
``src/aeo_quant/bridges/gemma4/linear_fp8.py:15-105``. The matmul is the
expert path's FP8 GEMM (``aeoq_fp8_quantize_rows_gather`` then
``aeoq_fp8_gemm``: per-row dynamic e4m3 input quantization, tcgen05
kind::f8f6f4, bf16((acc * sa[m]) * sb[n])) in place of ``torch._scaled_mm``;
the bias is added afterwards in bf16 as in the reference (:41-42).

The GEMM takes output widths in multiples of 128. A layer whose width is not
one (a Gemma-4 dense MLP of 2112, say) runs on a copy of its weight padded
with zero rows to the next multiple; the module keeps that copy beside its
parameters (rebuilt when the weight changes) and returns the first ``out``
columns.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import moe_ops

FP8_MAX = 448.0
_N_ALIGN = 128


def _padded(w_fp8: torch.Tensor, scale_w: torch.Tensor):
    N, K = w_fp8.shape
    Np = -(-N // _N_ALIGN) * _N_ALIGN
    wp = torch.zeros(Np, K, dtype=torch.uint8, device=w_fp8.device)
    wp[:N] = w_fp8.view(torch.uint8)
    sp = torch.zeros(1, Np, dtype=torch.float32, device=w_fp8.device)
    sp[0, :N] = scale_w.reshape(N).float()
    return wp.view(torch.float8_e4m3fn), sp


def fp8_linear(x_bf16: torch.Tensor, w_fp8: torch.Tensor, scale_w: torch.Tensor,
               bias: torch.Tensor | None = None, _padded_w=None) -> torch.Tensor:
    """(..., K) bf16 -> (..., N) bf16 (linear_fp8.py:15-45)."""
    N = w_fp8.shape[0]
    if N % _N_ALIGN:
        wp, sp = _padded_w if _padded_w is not None else _padded(w_fp8, scale_w)
        out = moe_ops.fp8_linear(x_bf16, wp, sp)[..., :N].contiguous()
    else:
        out = moe_ops.fp8_linear(x_bf16, w_fp8, scale_w)
    if bias is not None:
        out = out + bias
    return out


class LinearFP8(nn.Module):
    """Drop-in replacement for ``nn.Linear`` with FP8 weights
    (linear_fp8.py:48-105)."""

    weight: torch.Tensor
    weight_scale: torch.Tensor
    bias: torch.Tensor | None

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device=None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=torch.float8_e4m3fn, device=device),
                                   requires_grad=False)
        self.register_buffer("weight_scale", torch.empty(1, out_features, dtype=torch.float32, device=device))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, dtype=torch.bfloat16, device=device),
                                     requires_grad=False)
        else:
            self.bias = None
        self._pad_cache = None

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "LinearFP8":
        """Quantize an existing ``nn.Linear`` (linear_fp8.py:83-99): per-row
        e4m3 weights with bf16 scales, stored as a (1, out) fp32 buffer."""
        from ...gpu.quant import quantize_2d_to_fp8

        has_bias = linear.bias is not None
        mod = cls(linear.in_features, linear.out_features, bias=has_bias, device=linear.weight.device)
        w_fp8, scale_bf16 = quantize_2d_to_fp8(linear.weight.data.to(torch.bfloat16))
        mod.weight = nn.Parameter(w_fp8, requires_grad=False)
        mod.weight_scale = scale_bf16.squeeze(-1).unsqueeze(0).float().contiguous()
        if has_bias:
            mod.bias = nn.Parameter(linear.bias.data.to(torch.bfloat16), requires_grad=False)
        return mod

    def _pad(self):
        if self.out_features % _N_ALIGN == 0:
            return None
        key = (self.weight.data_ptr(), self.weight._version, self.weight_scale.data_ptr(),
               self.weight_scale._version)
        if self._pad_cache is None or self._pad_cache[0] != key:
            self._pad_cache = (key, _padded(self.weight, self.weight_scale))
        return self._pad_cache[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fp8_linear(x, self.weight, self.weight_scale, self.bias, _padded_w=self._pad())

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, dtype=float8_e4m3fn")
