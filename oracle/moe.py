"""CPU restatement of the Gemma-4 quantized expert forwards (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each function restates one reference forward line by line, keeping every
bf16 rounding point; only the GEMM calls are replaced by ``oracle.gemm``.

* ``nvfp4_experts_forward`` -> ``Gemma4TextExpertsNVFP4.forward``
  (aeo_quant ``src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:114-130``),
  with ``_decode_3d`` (:132-186) for one token and ``_prefill`` (:188-255)
  otherwise.
* ``fp8_experts_forward`` -> ``Gemma4TextExpertsFP8.forward``
  (``bridges/gemma4/modeling.py:110-146``).

Arrays: hidden (T,H) float32 holding bf16 values; top_k_index (T,k) int;
top_k_weights (T,k) float32 holding bf16 values.
"""
from __future__ import annotations

import numpy as np

from .gemm import fp8_scaled_mm, nvfp4_gemm, nvfp4_linear
from .numerics import F32, bf16, gelu_tanh
from .quant import quantize_fp8_activation_rows, quantize_nvfp4


class NVFP4Experts:
    """Buffers of ``Gemma4TextExpertsNVFP4`` (modeling_nvfp4.py:78-112)."""

    def __init__(self, gate_up_proj, gate_up_proj_scale, gate_up_proj_scale_2,
                 down_proj, down_proj_scale, down_proj_scale_2):
        self.gate_up_proj = np.asarray(gate_up_proj, np.uint8)
        self.gate_up_proj_scale = np.asarray(gate_up_proj_scale, np.uint8)
        self.gate_up_proj_scale_2 = F32(gate_up_proj_scale_2)
        self.down_proj = np.asarray(down_proj, np.uint8)
        self.down_proj_scale = np.asarray(down_proj_scale, np.uint8)
        self.down_proj_scale_2 = F32(down_proj_scale_2)
        self.num_experts = self.gate_up_proj.shape[0]
        self.intermediate = self.gate_up_proj.shape[1] // 2


def geglu(gate_up):
    """``act_fn(gate) * up`` in bf16 (modeling_nvfp4.py:161-162, :233-234)."""
    I = gate_up.shape[-1] // 2
    gate, up = gate_up[..., :I], gate_up[..., I:]
    return bf16(bf16(gelu_tanh(gate)) * up)


def nvfp4_decode_3d(m: NVFP4Experts, hidden, top_k_index, top_k_weights):
    """``_forward_decode_3d`` (modeling_nvfp4.py:132-186) for one token."""
    ids = np.asarray(top_k_index)[0]
    hp, hs, hts = quantize_nvfp4(hidden)                                   # :150-153
    gu = np.stack([nvfp4_gemm(hp, hs, hts, m.gate_up_proj[e], m.gate_up_proj_scale[e],
                              m.gate_up_proj_scale_2) for e in ids])        # :155-160 (k,1,2I)
    cur = geglu(gu)[:, 0, :]                                              # :161-162
    dp, ds, dts = quantize_nvfp4(cur)                                     # :164-172 shared ts
    down = np.stack([nvfp4_gemm(dp[j:j + 1], ds[j:j + 1], dts, m.down_proj[e],
                                m.down_proj_scale[e], m.down_proj_scale_2)
                     for j, e in enumerate(ids)])                         # :174-179 (k,1,H)
    w = np.asarray(top_k_weights, F32)[0][:, None, None]
    prod = bf16(down * w)                                                 # :183-184
    return bf16(prod.astype(np.float64).sum(0).astype(F32))


def nvfp4_prefill(m: NVFP4Experts, hidden, top_k_index, top_k_weights):
    """``_forward_prefill`` (modeling_nvfp4.py:188-255)."""
    hidden = np.asarray(hidden, F32)
    idx = np.asarray(top_k_index)
    wts = np.asarray(top_k_weights, F32)
    hp, hs, hts = quantize_nvfp4(hidden)                                   # :203-206
    final = np.zeros_like(hidden)
    for e in np.unique(idx):                                              # :209-218
        if e == m.num_experts:
            continue
        pos, tok = np.nonzero(idx.T == e)                                 # :222 (k,T) order
        gu = nvfp4_gemm(hp[tok], hs[tok], hts, m.gate_up_proj[e],
                        m.gate_up_proj_scale[e], m.gate_up_proj_scale_2)  # :225-232
        cur = geglu(gu)                                                   # :233-234
        d = nvfp4_linear(cur, m.down_proj[e], m.down_proj_scale[e],
                         m.down_proj_scale_2)                             # :239-244 per-expert ts
        d = bf16(d * wts[tok, pos][:, None])                              # :247-249
        final[tok] = bf16(final[tok] + d)                                 # :250-253
    return final


def nvfp4_experts_forward(m: NVFP4Experts, hidden, top_k_index, top_k_weights):
    """Shape dispatch of ``forward`` (modeling_nvfp4.py:124-130)."""
    if np.asarray(hidden).shape[0] == 1:
        return nvfp4_decode_3d(m, hidden, top_k_index, top_k_weights)
    return nvfp4_prefill(m, hidden, top_k_index, top_k_weights)


class FP8Experts:
    """Buffers of ``Gemma4TextExpertsFP8`` after ``_preconvert_fp8_scales``
    (modeling.py:64-87, loader.py:47-64): e4m3 codes and (E,1,N) f32 scales."""

    def __init__(self, gate_up_proj, gate_up_proj_scale, down_proj, down_proj_scale):
        self.gate_up_proj = np.asarray(gate_up_proj, np.uint8)
        self.gate_up_proj_scale = np.asarray(gate_up_proj_scale, F32).reshape(
            self.gate_up_proj.shape[0], 1, -1)
        self.down_proj = np.asarray(down_proj, np.uint8)
        self.down_proj_scale = np.asarray(down_proj_scale, F32).reshape(
            self.down_proj.shape[0], 1, -1)
        self.num_experts = self.gate_up_proj.shape[0]


def fp8_linear(x, w_codes, sb):
    """``_fp8_linear`` (modeling.py:89-108)."""
    q, sa = quantize_fp8_activation_rows(x)
    return fp8_scaled_mm(q, sa, w_codes, sb)


def fp8_experts_forward(m: FP8Experts, hidden, top_k_index, top_k_weights):
    """``Gemma4TextExpertsFP8.forward`` (modeling.py:110-146)."""
    hidden = np.asarray(hidden, F32)
    idx = np.asarray(top_k_index)
    wts = np.asarray(top_k_weights, F32)
    final = np.zeros_like(hidden)
    for e in np.unique(idx):
        if e == m.num_experts:
            continue
        pos, tok = np.nonzero(idx.T == e)
        gu = fp8_linear(hidden[tok], m.gate_up_proj[e], m.gate_up_proj_scale[e])
        cur = geglu(gu)
        d = fp8_linear(cur, m.down_proj[e], m.down_proj_scale[e])
        d = bf16(d * wts[tok, pos][:, None])
        final[tok] = bf16(final[tok] + d)
    return final
