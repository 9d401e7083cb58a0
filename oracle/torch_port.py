"""torch restatement of the oracle's NVFP4 expert forward (any device).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): it serves as the
CPU baseline that ``bench.py`` times on the host cores and as a GPU-speed
checker for the random-init decoder stack in ``tests/``. It is pinned to the
numpy oracle by ``tests/test_torch_port.py`` (quantizer bytes bit for bit,
forwards within the output tolerance).

It follows the same reference lines as ``oracle/quant.py`` and
``oracle/moe.py``:

* ``quantize_nvfp4`` -> ``quantize_2d_to_nvfp4`` (aeo_quant
  ``src/aeo_quant/gpu/quant.py:138-185``, :215-230): global amax, tensor
  scale in the input dtype, per-16 e4m3 block scale, E2M1 binning by
  midpoints with ties to the smaller magnitude, high nibble = even k;
* ``nvfp4_gemm`` -> the ``tl.dot_scaled`` contract of
  ``nvfp4_linear_prequantized`` (``gpu/nvfp4_matmul.py:399-519``): exact
  block-scaled operands, float32 products summed in float32 (float64 with
  ``exact=True``), times alpha = f32(a_ts) * f32(w_ts), rounded once to bf16;
* ``decode_3d`` / ``prefill`` -> ``Gemma4TextExpertsNVFP4._forward_decode_3d``
  / ``_forward_prefill`` (``bridges/gemma4/modeling_nvfp4.py:132-186``,
  :188-255), with every bf16 rounding point.

The difference from the numpy oracle is the accumulation: a float32 matmul
(BLAS order) instead of one float64 dot product rounded to float32.
"""
from __future__ import annotations

import torch

_FP4 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
_BOUNDS = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
_LUT: dict = {}


def _lut(device):
    t = _LUT.get(device)
    if t is None:
        t = _LUT[device] = torch.tensor(_FP4, dtype=torch.float32, device=device)
    return t


def tensor_scale(amax: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """ts = max(amax / 2688, 1e-12) rounded to the input dtype (quant.py:167-168)."""
    ts = (amax.to(torch.float32) / 2688.0).to(dtype)
    floor = torch.tensor(1e-12, dtype=torch.float32).to(dtype).to(amax.device)
    return torch.maximum(ts, floor).to(torch.float32)


def quantize_nvfp4(x: torch.Tensor, ts: torch.Tensor | None = None):
    """(packed u8 [..., K/2], e4m3 codes u8 [..., K/16], ts f32 0-d) of a
    bf16 tensor ``x[..., K]`` (quant.py:138-185)."""
    xf = x.to(torch.float32)
    K = xf.shape[-1]
    if ts is None:
        amax = xf.abs().amax() if xf.numel() else torch.zeros((), device=xf.device)
        ts = tensor_scale(amax, x.dtype)
    w = xf / ts                                                             # :169
    blocks = w.reshape(*xf.shape[:-1], K // 16, 16)
    bmax = torch.clamp(blocks.abs().amax(-1, keepdim=True), min=1e-8)     # :173
    sf = (bmax / 6.0).to(torch.float8_e4m3fn)                             # :174
    q = blocks / sf.to(torch.float32)                                     # :177
    q = torch.where(torch.isnan(q), q, q.clamp(-6.0, 6.0))
    mag = q.abs()
    idx = torch.zeros(q.shape, dtype=torch.uint8, device=q.device)
    for b in _BOUNDS:
        idx += (mag > b).to(torch.uint8)
    idx = torch.where(torch.isnan(q), torch.full_like(idx, 7), idx)
    nib = (idx | ((q < 0).to(torch.uint8) << 3)).reshape(*xf.shape[:-1], K // 2, 2)
    packed = (nib[..., 0] << 4) | nib[..., 1]                             # :180-183
    return packed, sf.view(torch.uint8).reshape(*xf.shape[:-1], K // 16), ts


def dequant_unscaled(packed: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    """Exact block-scaled operand: E2M1 value x e4m3 block scale, float32."""
    hi, lo = packed >> 4, packed & 0xF
    nib = torch.stack([hi, lo], -1).reshape(*packed.shape[:-1], packed.shape[-1] * 2).long()
    v = _lut(packed.device)[nib]
    K = v.shape[-1]
    s = sf.view(torch.float8_e4m3fn).to(torch.float32)
    return (v.reshape(*v.shape[:-1], K // 16, 16) * s[..., None]).reshape(*v.shape[:-1], K)


def nvfp4_gemm(a_packed, a_sf, a_ts, w_packed, w_sf, w_ts, exact: bool = False) -> torch.Tensor:
    """bf16(alpha * A W^T) over exact block-scaled operands (nvfp4_matmul.py:315-325, :437)."""
    dt = torch.float64 if exact else torch.float32
    a = dequant_unscaled(a_packed, a_sf).to(dt)
    w = dequant_unscaled(w_packed, w_sf).to(dt)
    acc = (a @ w.T).to(torch.float32)
    alpha = torch.as_tensor(a_ts, dtype=torch.float32) * torch.as_tensor(w_ts, dtype=torch.float32)
    return (acc * alpha.to(acc.device)).to(torch.bfloat16)


def geglu(gate_up: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(gelu_tanh(gate)) * up) on bf16 values (modeling_nvfp4.py:161-162)."""
    I = gate_up.shape[-1] // 2
    g = gate_up[..., :I].to(torch.float32)
    u = gate_up[..., I:].to(torch.float32)
    beta = 0.7978845608028654   # sqrt(2/pi)
    ge = 0.5 * g * (1.0 + torch.tanh(beta * (g + 0.044715 * (g * g * g))))
    return (ge.to(torch.bfloat16).to(torch.float32) * u).to(torch.bfloat16)


class Experts:
    """The reference buffers of ``Gemma4TextExpertsNVFP4`` (modeling_nvfp4.py:78-112)."""

    def __init__(self, gate_up, gate_up_sf, gate_up_ts, down, down_sf, down_ts):
        self.gu, self.gu_sf, self.gu_ts = gate_up, gate_up_sf.view(torch.uint8), gate_up_ts
        self.dw, self.dw_sf, self.dw_ts = down, down_sf.view(torch.uint8), down_ts
        self.num_experts = gate_up.shape[0]


def decode_3d(m: Experts, hidden, top_k_index, top_k_weights, exact=False):
    """``_forward_decode_3d`` (modeling_nvfp4.py:132-186) for one token."""
    ids = top_k_index.reshape(-1).tolist()
    hp, hs, hts = quantize_nvfp4(hidden)                                  # :150-153
    gu = torch.stack([nvfp4_gemm(hp, hs, hts, m.gu[e], m.gu_sf[e], m.gu_ts, exact) for e in ids])
    cur = geglu(gu)[:, 0, :]                                              # :161-162
    dp, ds, dts = quantize_nvfp4(cur)                                     # :164-172 shared ts
    down = torch.stack([nvfp4_gemm(dp[j:j + 1], ds[j:j + 1], dts, m.dw[e], m.dw_sf[e], m.dw_ts, exact)
                        for j, e in enumerate(ids)])                      # :174-179
    w = top_k_weights.reshape(-1).to(torch.float32)[:, None, None]
    prod = (down.to(torch.float32) * w).to(torch.bfloat16)                # :183-184
    return prod.to(torch.float64).sum(0).to(torch.float32).to(torch.bfloat16)


def prefill(m: Experts, hidden, top_k_index, top_k_weights, exact=False):
    """``_forward_prefill`` (modeling_nvfp4.py:188-255)."""
    hp, hs, hts = quantize_nvfp4(hidden)                                  # :203-206
    final = torch.zeros(hidden.shape, dtype=torch.bfloat16, device=hidden.device)
    idx = top_k_index
    wts = top_k_weights.to(torch.float32)
    for e in torch.unique(idx).tolist():                                  # :209-218
        if e < 0 or e >= m.num_experts:
            continue
        pos, tok = torch.nonzero(idx.T == e, as_tuple=True)              # :222 (k,T) order
        gu = nvfp4_gemm(hp[tok], hs[tok], hts, m.gu[e], m.gu_sf[e], m.gu_ts, exact)   # :225-232
        cur = geglu(gu)                                                   # :233-234
        dp, ds, dts = quantize_nvfp4(cur)                                 # :239-244 per-expert ts
        d = nvfp4_gemm(dp, ds, dts, m.dw[e], m.dw_sf[e], m.dw_ts, exact)
        d = (d.to(torch.float32) * wts[tok, pos][:, None]).to(torch.bfloat16)        # :247-249
        final[tok] = (final[tok].to(torch.float32) + d.to(torch.float32)).to(torch.bfloat16)   # :250-253
    return final


def forward(m: Experts, hidden, top_k_index, top_k_weights, exact=False):
    """Shape dispatch of ``forward`` (modeling_nvfp4.py:124-130)."""
    if hidden.shape[0] == 1:
        return decode_3d(m, hidden, top_k_index, top_k_weights, exact)
    return prefill(m, hidden, top_k_index, top_k_weights, exact)
