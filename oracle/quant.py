"""CPU restatement of the NVFP4 and FP8 quantizers (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Each function follows
the aeo_quant reference line by line; citations are to
``src/aeo_quant/gpu/quant.py`` and ``src/aeo_quant/bridges/gemma4/modeling.py``.

Inputs are float32 arrays that already hold values of the input dtype
(``dtype="bf16"`` means every element is a bf16 value). Outputs:
packed FP4 bytes (uint8), e4m3 scale codes (uint8), and tensor scales as
float32 values of the input dtype.
"""
from __future__ import annotations

import numpy as np

from .numerics import (F32, FP4_E2M1_MAX, FP8_E4M3_MAX, NVFP4_BLOCK, bf16,
                       e4m3_decode, e4m3_encode, fp4_nibble)


def _round_to(dtype: str, x):
    x = np.asarray(x, dtype=F32)
    if dtype == "bf16":
        return bf16(x)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(F32)
    raise ValueError(dtype)


def nvfp4_tensor_scale(amax, dtype: str = "bf16"):
    """ts = clamp(amax / (6*448), min=1e-12) in the input dtype (quant.py:167-168)."""
    ts = _round_to(dtype, F32(amax) / F32(FP4_E2M1_MAX * FP8_E4M3_MAX))
    floor = _round_to(dtype, F32(1e-12))
    return np.maximum(ts, floor).astype(F32)


def quantize_nvfp4(x, dtype: str = "bf16", ts=None):
    """Two-level NVFP4 quantization of ``x[..., K]`` (quant.py:138-185).

    ``ts`` may be passed to reuse a tensor scale; by default it is derived
    from the global amax of ``x`` exactly as the reference does.
    Returns ``(packed uint8 [..., K/2], scale codes uint8 [..., K/16], ts)``.
    """
    x = np.asarray(x, dtype=F32)
    K = x.shape[-1]
    if K % NVFP4_BLOCK:
        raise ValueError(f"in_dim ({K}) must be divisible by block_size ({NVFP4_BLOCK})")
    if ts is None:
        amax = np.max(np.abs(x)) if x.size else F32(0.0)
        ts = nvfp4_tensor_scale(amax, dtype)
    ts = F32(ts)
    with np.errstate(divide="ignore", invalid="ignore"):
        w = (x / ts).astype(F32)                                      # :169
        blocks = w.reshape(*x.shape[:-1], K // NVFP4_BLOCK, NVFP4_BLOCK)
        bmax = np.maximum(np.abs(blocks).max(axis=-1, keepdims=True), F32(1e-8))  # :173
        sf = e4m3_encode((bmax / F32(FP4_E2M1_MAX)).astype(F32))      # :174
        q = (blocks / e4m3_decode(sf)).astype(F32)                    # :177
    q = np.where(np.isnan(q), q, np.clip(q, -FP4_E2M1_MAX, FP4_E2M1_MAX))
    nib = fp4_nibble(q).reshape(*x.shape[:-1], K // 2, 2)
    packed = ((nib[..., 0] << 4) | nib[..., 1]).astype(np.uint8)      # :180-183
    return packed, sf.reshape(*x.shape[:-1], K // NVFP4_BLOCK), F32(ts)


def dequant_nvfp4_unscaled(packed, sf):
    """FP4 value x e4m3 block scale in float32, without the tensor scale.

    Every product here is exact in float32 (a 2-bit by 4-bit mantissa), so
    this is the exact operand the block-scaled MMA sees. The nibble order
    follows the reference packing: high nibble = even k (quant.py:201-204).
    """
    from .numerics import FP4_LUT
    packed = np.asarray(packed, dtype=np.uint8)
    hi = packed >> 4
    lo = packed & 0xF
    nib = np.stack([hi, lo], axis=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    vals = FP4_LUT[nib]
    K = vals.shape[-1]
    vals = vals.reshape(*vals.shape[:-1], K // NVFP4_BLOCK, NVFP4_BLOCK)
    vals = vals * e4m3_decode(sf)[..., None]
    return vals.reshape(*packed.shape[:-1], K).astype(F32)


def dequant_nvfp4(packed, sf, ts):
    """``dequant_3d_from_nvfp4`` (quant.py:188-212): value*bs*ts -> bf16."""
    return bf16(dequant_nvfp4_unscaled(packed, sf) * F32(ts))


def quantize_fp8_rows(w):
    """Per-row max-abs FP8 weight quant (quant.py:51-75 / :85-106).

    Returns ``(e4m3 codes [..., K], bf16 scale values [..., 1])``.
    """
    w = np.asarray(w, dtype=F32)
    amax = np.abs(w).max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        s = bf16(amax / F32(FP8_E4M3_MAX))
        s = np.where(np.isnan(s), s, np.maximum(s, bf16(F32(1e-8))))
    with np.errstate(divide="ignore", invalid="ignore"):
        q = e4m3_encode((w / s).astype(F32))
    return q, s.astype(F32)


def quantize_fp8_activation_rows(x):
    """Per-row dynamic FP8 activation quant inside ``_fp8_linear``
    (bridges/gemma4/modeling.py:101-104).

    amax is taken on the bf16 values and clamped at bf16(1e-4); the scale is
    the float32 quotient amax/448. Returns ``(codes, scale f32 [..., 1])``.
    """
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).max(axis=-1, keepdims=True) if x.shape[-1] else np.zeros(x.shape[:-1] + (1,), F32)
    amax = np.maximum(amax, bf16(F32(1e-4)))
    sa = (amax / F32(FP8_E4M3_MAX)).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = e4m3_encode((x / sa).astype(F32))
    return q, sa
