"""Bit-level number formats used by the quantized MoE expert path (numpy).

TEST INFRASTRUCTURE ONLY. This package is the CPU checker for the CUDA
library: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may import it. The product path never routes through it.

The reference computes with torch dtypes (``bfloat16``, ``float8_e4m3fn``)
and a 16-entry FP4 E2M1 table (aeo_quant ``src/aeo_quant/gpu/quant.py:15-27``).
numpy has none of these, so this module restates each format from its
definition:

* bf16: the upper 16 bits of an IEEE binary32, rounded to nearest-even.
* float8_e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits, no infinity,
  the all-ones pattern ``S.1111.111`` is NaN, largest finite 448. torch's
  conversion rounds to nearest-even and yields NaN for anything that rounds
  past 448 (i.e. magnitudes above 464, and 464 itself ties down to 448).
* FP4 E2M1: sign-magnitude nibble, magnitudes {0,.5,1,1.5,2,3,4,6}.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# FP4 E2M1 magnitudes by nibble (quant.py:24-27). Nibble 8 is -0.0.
FP4_LUT = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=F32)
# Midpoints between adjacent magnitudes (quant.py:21).
FP4_BOUNDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=F32)

FP8_E4M3_MAX = 448.0
FP4_E2M1_MAX = 6.0
NVFP4_BLOCK = 16


# ----------------------------------------------------------------------------
# bfloat16
# ----------------------------------------------------------------------------
def bf16_bits(x) -> np.ndarray:
    """float32 -> uint16 bf16 pattern, round-to-nearest-even, NaN -> 0x7FC0."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    b = x.view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    r = ((b + 0x7FFF + lsb) >> 16).astype(np.uint32) & 0xFFFF
    nan = np.isnan(x)
    r = np.where(nan, (b >> 16).astype(np.uint32) | 0x40, r)
    return r.astype(np.uint16)


def bf16_from_bits(h) -> np.ndarray:
    h = np.asarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(F32)


def bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (kept as float32)."""
    return bf16_from_bits(bf16_bits(x))


# ----------------------------------------------------------------------------
# float8_e4m3fn
# ----------------------------------------------------------------------------
def e4m3_encode(x) -> np.ndarray:
    """float32 -> uint8 e4m3fn code with torch's ``.to(float8_e4m3fn)`` rules."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F32))
    bits = x.view(np.uint32)
    sign = ((bits >> 31) & 1).astype(np.uint32) << 7
    a = np.abs(x)
    abits = a.view(np.uint32).astype(np.int64)
    out = np.zeros(x.shape, dtype=np.int64)
    # normal range: |x| >= 2^-6
    normal = a >= F32(2.0 ** -6)
    r = (abits + 0x7FFFF + ((abits >> 20) & 1)) >> 20   # (exp32 << 3 | mant3), RNE
    code_n = r - ((127 - 7) << 3)
    out = np.where(normal, code_n, out)
    # subnormal range: k * 2^-9, k in [0, 8] (8 is the smallest normal)
    with np.errstate(invalid="ignore"):
        k = np.rint(np.where(np.isfinite(a), a, 0).astype(np.float64) * 512.0).astype(np.int64)
    out = np.where(~normal, k, out)
    # overflow past 448 -> NaN code; NaN/inf -> NaN code
    out = np.where((out > 0x7E) | ~np.isfinite(x), 0x7F, out)
    return (out.astype(np.uint32) | sign).astype(np.uint8)


def e4m3_decode(c) -> np.ndarray:
    c = np.asarray(c, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    mag = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    mag = np.where((e == 15) & (m == 7), np.nan, mag)
    return (s * mag).astype(F32)


# ----------------------------------------------------------------------------
# FP4 E2M1
# ----------------------------------------------------------------------------
def fp4_nibble(x) -> np.ndarray:
    """Nearest E2M1 nibble with ties toward the smaller magnitude; NaN -> 7.

    Restates ``_round_to_fp4_e2m1`` (quant.py:121-130): the magnitude index is
    the count of midpoints strictly below |x| (``searchsorted``, right=False),
    NaN sorts past every bound, and the sign bit is ``x < 0``.
    """
    x = np.asarray(x, dtype=F32)
    mag = np.abs(x)
    idx = np.zeros(x.shape, dtype=np.uint8)
    for b in FP4_BOUNDS:
        idx += (mag > b).astype(np.uint8)
    idx = np.where(np.isnan(x), np.uint8(7), idx)
    sign = (x < 0).astype(np.uint8) << 3
    return (sign | idx).astype(np.uint8)


def gelu_tanh(x) -> np.ndarray:
    """tanh-approximated GELU evaluated in float32 (Gemma4 ``gelu_pytorch_tanh``)."""
    x = np.asarray(x, dtype=F32)
    k_beta = F32(np.sqrt(2.0) * (2.0 / np.sqrt(np.pi)) * 0.5)
    k_kappa = F32(0.044715)
    inner = k_beta * (x + k_kappa * (x * x * x))
    return (F32(0.5) * x * (F32(1.0) + np.tanh(inner).astype(F32))).astype(F32)
