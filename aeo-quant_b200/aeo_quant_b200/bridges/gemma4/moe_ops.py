"""Host side of the fused expert forwards: shape checks, workspace, C-ABI calls.

Shared by ``Gemma4TextExpertsNVFP4`` and ``Gemma4TextExpertsFP8``. Each
function restates one reference forward; the arithmetic is in the sm_100a
library.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ... import _capi as A
from ...gpu import nvfp4_matmul as NM
from ...gpu.quant import quantize_2d_to_nvfp4


_FUSED_WS: dict = {}


def _fused_workspace(lib, device, k, H, I):
    """Zero-initialised workspace of the cooperative decode kernel, one per
    (device, shape). The kernel leaves its counters zero on exit, so the
    buffer is reused by every stream-ordered call (not by overlapping ones)."""
    key = (device.index, k, H, I)
    ws = _FUSED_WS.get(key)
    if ws is None:
        n = lib.aeoq_moe_nvfp4_decode_fused_workspace_size(k, H, I)
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _FUSED_WS[key] = ws
    return ws


def nvfp4_decode(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, fused=None):
    """One-token forward (modeling_nvfp4.py:132-186): one cooperative kernel
    when the shape fits its shared-memory plan, else three chained launches."""
    A.require_cuda(hidden, top_k_index, top_k_weights, gu, dw)
    lib = A.load()
    if hidden.dtype != torch.bfloat16:
        raise ValueError(f"hidden_states must be bfloat16, got {hidden.dtype}")
    E, two_i, h_half = gu.shape
    H, I = h_half * 2, two_i // 2
    if hidden.shape[-1] != H:
        raise ValueError(f"hidden size {hidden.shape[-1]} != expert hidden size {H}")
    k = top_k_index.shape[-1]
    hidden = hidden.contiguous()
    idx = top_k_index.reshape(-1)[:k].contiguous()
    w = top_k_weights.reshape(-1)[:k].to(torch.bfloat16).contiguous()
    out = torch.empty(1, H, dtype=torch.bfloat16, device=hidden.device)
    if fused is None:
        fused = bool(lib.aeoq_moe_nvfp4_decode_fused_supported(k, H, I))
    if fused:
        ws = _fused_workspace(lib, hidden.device, k, H, I)
        fn, ws_n = lib.aeoq_moe_nvfp4_decode_fused, ws.numel()
    else:
        ws_n = lib.aeoq_moe_nvfp4_decode_workspace_size(k, H, I)
        ws = torch.empty(ws_n, dtype=torch.uint8, device=hidden.device)
        fn = lib.aeoq_moe_nvfp4_decode
    A.check(fn(
        hidden.data_ptr(), idx.data_ptr(), A.dtype_code(idx.dtype), w.data_ptr(), k,
        gu.data_ptr(), gu_sf.data_ptr(), gu_ts.data_ptr(), A.dtype_code(gu_ts.dtype),
        dw.data_ptr(), dw_sf.data_ptr(), dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype),
        E, H, I, out.data_ptr(), ws.data_ptr(), ws_n, A.stream_ptr(hidden.device)))
    return out


def nvfp4_prefill(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, num_experts):
    """Many-token forward (modeling_nvfp4.py:188-255)."""
    h_packed, h_block_scale, h_tensor_scale = quantize_2d_to_nvfp4(hidden)
    final_hidden_states = torch.zeros_like(hidden)
    with torch.no_grad():
        expert_mask = nn.functional.one_hot(top_k_index, num_classes=num_experts).permute(2, 1, 0)
        expert_hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero()
    I = gu.shape[1] // 2
    for expert_idx in expert_hit:
        expert_idx = expert_idx[0]
        if expert_idx == num_experts:
            continue
        top_k_pos, token_idx = torch.where(expert_mask[expert_idx])
        gate_up = NM.nvfp4_linear_prequantized(
            h_packed[token_idx], h_block_scale[token_idx], h_tensor_scale,
            gu[expert_idx], gu_sf[expert_idx], gu_ts)
        gate, up = gate_up[:, :I], gate_up[:, I:]
        cur = nn.functional.gelu(gate, approximate="tanh") * up
        cur = NM.nvfp4_linear(cur, dw[expert_idx], dw_sf[expert_idx], dw_ts)
        cur *= top_k_weights[token_idx, top_k_pos, None]
        final_hidden_states.index_add_(0, token_idx, cur.to(final_hidden_states.dtype))
    return final_hidden_states
