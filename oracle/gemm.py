"""CPU restatement of the block-scaled NVFP4 and rowwise FP8 GEMMs (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference's GEMM arithmetic lives in third-party code that is not under
the reference tree: Triton 3.6.0 ``tl.dot_scaled`` (aeo_quant
``src/aeo_quant/gpu/nvfp4_matmul.py:129,226,313``) and cuBLASLt behind torch
2.11 ``torch._scaled_mm`` (``bridges/gemma4/modeling.py:105-108``). Their
published contract is restated here:

* NVFP4: ``C = bf16(alpha * sum_k (a_k*sA)(w_k*sW))`` with ``alpha =
  f32(a_ts)*f32(w_ts)`` (nvfp4_matmul.py:315-325, :437). The block-scaled
  operands are exact in float32; the dot product is taken in float64 and
  rounded once to float32 (a tighter bound than any fp32 accumulation order).
* FP8 rowwise: ``C = bf16(sum_k q_x q_w * sa[m] * sb[n])``.
"""
from __future__ import annotations

import numpy as np

from .numerics import F32, bf16, e4m3_decode
from .quant import dequant_nvfp4_unscaled, quantize_nvfp4


def nvfp4_gemm(a_packed, a_sf, a_ts, w_packed, w_sf, w_ts, out="bf16"):
    """``nvfp4_linear_prequantized`` semantics (nvfp4_matmul.py:399-519).

    ``out="f32"`` returns the float32 epilogue value (the ``out_dtype=float32``
    path of the reference launchers) instead of rounding it to bf16.
    """
    a = dequant_nvfp4_unscaled(a_packed, a_sf).astype(np.float64)
    w = dequant_nvfp4_unscaled(w_packed, w_sf).astype(np.float64)
    acc = (a @ w.T).astype(F32)
    alpha = F32(F32(a_ts) * F32(w_ts))
    y = (acc * alpha).astype(F32)
    return y if out == "f32" else bf16(y)


def nvfp4_linear(x, w_packed, w_sf, w_ts, dtype: str = "bf16"):
    """``nvfp4_linear`` (nvfp4_matmul.py:357-396): quantize x, then GEMM."""
    x = np.asarray(x, dtype=F32)
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    ap, asf, ats = quantize_nvfp4(x2, dtype)
    out = nvfp4_gemm(ap, asf, ats, w_packed, w_sf, w_ts)
    return out.reshape(*shp[:-1], out.shape[-1])


def nvfp4_gemm_3d(a_packed, a_sf, a_ts, w_packed, w_sf, w_ts, expert_ids=None):
    """``nvfp4_linear_3d_prequantized`` / ``nvfp4_linear_3d_gather``
    (nvfp4_matmul.py:522-686, :689-864): 2D activation is shared by every
    expert, 3D activation is per selected expert. Returns ``(E_sel, M, N)``.
    """
    ids = np.arange(w_packed.shape[0]) if expert_ids is None else np.asarray(expert_ids)
    outs = []
    for j, e in enumerate(ids):
        ap = a_packed if a_packed.ndim == 2 else a_packed[j]
        asf = a_sf if a_sf.ndim == 2 else a_sf[j]
        outs.append(nvfp4_gemm(ap, asf, a_ts, w_packed[e], w_sf[e], w_ts))
    return np.stack(outs, 0)


def fp8_scaled_mm(q_x, sa, q_w, sb):
    """Rowwise-scaled FP8 GEMM: ``bf16(acc * sa[m] * sb[n])``.

    ``q_x`` (M,K) and ``q_w`` (N,K) are e4m3 codes, ``sa`` (M,1) and ``sb``
    (N,) or (1,N) float32.
    """
    x = e4m3_decode(q_x).astype(np.float64)
    w = e4m3_decode(q_w).astype(np.float64)
    acc = (x @ w.T).astype(F32)
    sb = np.asarray(sb, F32).reshape(1, -1)
    return bf16((acc * np.asarray(sa, F32).reshape(-1, 1)).astype(F32) * sb)
