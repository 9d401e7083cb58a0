"""FP8 and NVFP4 quantizers on B200 — drop-in for ``aeo_quant.gpu.quant``.

Same names, signatures, return dtypes/shapes and ``ValueError`` messages as
aeo_quant ``src/aeo_quant/gpu/quant.py``; the arithmetic runs in the
sm_100a library (``csrc/quant.cu``) and is bit-exact with the reference:

* NVFP4 (quant.py:138-230): per-tensor scale ``clamp(amax/2688, 1e-12)`` in
  the input dtype, e4m3 scale per 16 along the last dim, E2M1 nibbles with
  ties toward the smaller magnitude, two per byte, high nibble first.
* FP8 (quant.py:51-106): per-row ``clamp(amax/448, 1e-8)`` scale in bf16.

Only CUDA tensors are accepted; there is no CPU path.
"""
from __future__ import annotations

import torch

from .. import _capi as A

FP8_E4M3_MAX = 448.0
FP4_E2M1_MAX = 6.0
NVFP4_BLOCK_SIZE = 16


def _rows_view(x: torch.Tensor) -> torch.Tensor:
    K = x.shape[-1]
    x2 = x.reshape(-1, K) if x.ndim != 2 else x
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _nvfp4_quantize_rows(x2: torch.Tensor, ts_in: torch.Tensor | None = None):
    """Quantize a (rows, K) tensor; returns (packed, block_scale, ts)."""
    A.require_cuda(x2)
    lib = A.load()
    rows, K = x2.shape
    dev = x2.device
    packed = torch.empty(rows, K // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(rows, K // NVFP4_BLOCK_SIZE, dtype=torch.float8_e4m3fn, device=dev)
    st = A.stream_ptr(dev)
    dt = A.dtype_code(x2.dtype)
    ld = x2.stride(0) if rows > 1 else K
    if ts_in is not None:
        A.check(lib.aeoq_nvfp4_quantize_with_scale(x2.data_ptr(), dt, rows, K, ld, ts_in.data_ptr(),
                                                   packed.data_ptr(), sf.data_ptr(), st))
        return packed, sf, ts_in
    ts = torch.empty((), dtype=x2.dtype, device=dev)
    ws_n = lib.aeoq_nvfp4_quantize_workspace_size(rows, K)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    A.check(lib.aeoq_nvfp4_quantize(x2.data_ptr(), dt, rows, K, ld, packed.data_ptr(), sf.data_ptr(),
                                    ts.data_ptr(), ws.data_ptr(), ws_n, st))
    return packed, sf, ts


def _require_block16(block_size: int) -> None:
    if block_size != NVFP4_BLOCK_SIZE:
        raise ValueError(f"block_size={block_size} is not supported: the NVFP4 kernels use "
                         f"{NVFP4_BLOCK_SIZE}-element micro-blocks")


def quantize_3d_to_fp8(weight_bf16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-(expert, output_channel) max-abs FP8 quant (quant.py:51-75).

    Returns ``(weight_fp8 (E,out,in) float8_e4m3fn, scale_bf16 (E,out,1) bfloat16)``.
    """
    if weight_bf16.ndim != 3:
        raise ValueError(
            f"quantize_3d_to_fp8 expects a 3D tensor (num_experts, out_dim, in_dim); "
            f"got shape {tuple(weight_bf16.shape)}"
        )
    q, s = _fp8_rows(weight_bf16, A.FP8_WEIGHT)
    return q, s


def quantize_2d_to_fp8(weight_bf16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-row max-abs FP8 quant (quant.py:85-106)."""
    if weight_bf16.ndim != 2:
        raise ValueError(
            f"quantize_2d_to_fp8 expects a 2D tensor (out_dim, in_dim); "
            f"got shape {tuple(weight_bf16.shape)}"
        )
    return _fp8_rows(weight_bf16, A.FP8_WEIGHT)


def _fp8_rows(x: torch.Tensor, mode: int):
    A.require_cuda(x)
    lib = A.load()
    x2 = _rows_view(x)
    rows, K = x2.shape
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    sdt = torch.bfloat16 if mode == A.FP8_WEIGHT else torch.float32
    s = torch.empty(*x.shape[:-1], 1, dtype=sdt, device=x.device)
    ld = x2.stride(0) if rows > 1 else K
    A.check(lib.aeoq_fp8_quantize_rows(x2.data_ptr(), A.dtype_code(x2.dtype), rows, K, ld, q.data_ptr(), K,
                                       s.data_ptr(), mode, A.stream_ptr(x.device)))
    return q, s


def quantize_fp8_activation_rows(x_bf16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row dynamic FP8 activation quant of ``_fp8_linear``
    (bridges/gemma4/modeling.py:101-104): returns ``(x_fp8, x_scale (M,1) f32)``."""
    return _fp8_rows(x_bf16, A.FP8_ACTIVATION)


def dequantize_3d_from_fp8(weight_fp8: torch.Tensor, scale_bf16: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`quantize_3d_to_fp8` for testing/validation only (quant.py:78-82)."""
    return weight_fp8.to(torch.bfloat16) * scale_bf16


def dequantize_2d_from_fp8(weight_fp8: torch.Tensor, scale_bf16: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`quantize_2d_to_fp8` for testing/validation only (quant.py:109-113)."""
    return weight_fp8.to(torch.bfloat16) * scale_bf16


def quantize_3d_to_nvfp4(
    weight_bf16: torch.Tensor, block_size: int = NVFP4_BLOCK_SIZE
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Two-level NVFP4 quantization of a 3D tensor (quant.py:138-185).

    Returns ``(packed (E,out,in/2) uint8, block_scale (E,out,in/16) float8_e4m3fn,
    tensor_scale 0-d in the input dtype)``.
    """
    if weight_bf16.ndim != 3:
        raise ValueError(
            f"quantize_3d_to_nvfp4 expects a 3D tensor (E, out_dim, in_dim); "
            f"got shape {tuple(weight_bf16.shape)}"
        )
    E, out_dim, in_dim = weight_bf16.shape
    if in_dim % block_size != 0:
        raise ValueError(
            f"in_dim ({in_dim}) must be divisible by block_size ({block_size})"
        )
    _require_block16(block_size)
    p, s, t = _nvfp4_quantize_rows(_rows_view(weight_bf16))
    return p.reshape(E, out_dim, in_dim // 2), s.reshape(E, out_dim, in_dim // block_size), t


def quantize_2d_to_nvfp4(
    weight_bf16: torch.Tensor, block_size: int = NVFP4_BLOCK_SIZE
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Two-level NVFP4 quantization of a 2D tensor (quant.py:215-230)."""
    if weight_bf16.ndim != 2:
        raise ValueError(
            f"quantize_2d_to_nvfp4 expects a 2D tensor (out_dim, in_dim); "
            f"got shape {tuple(weight_bf16.shape)}"
        )
    packed, block_scale, tensor_scale = quantize_3d_to_nvfp4(weight_bf16.unsqueeze(0), block_size)
    return packed.squeeze(0), block_scale.squeeze(0), tensor_scale


def _nvfp4_dequant(packed: torch.Tensor, block_scale: torch.Tensor, tensor_scale: torch.Tensor):
    A.require_cuda(packed, block_scale, tensor_scale)
    lib = A.load()
    K = packed.shape[-1] * 2
    p2 = packed.reshape(-1, K // 2).contiguous()
    s2 = block_scale.reshape(-1, K // NVFP4_BLOCK_SIZE).contiguous()
    out = torch.empty(*packed.shape[:-1], K, dtype=torch.bfloat16, device=packed.device)
    A.check(lib.aeoq_nvfp4_dequantize(p2.data_ptr(), s2.data_ptr(), tensor_scale.data_ptr(),
                                      A.dtype_code(tensor_scale.dtype), p2.shape[0], K, out.data_ptr(),
                                      A.stream_ptr(packed.device)))
    return out


def dequant_3d_from_nvfp4(packed_uint8, block_scale_fp8, tensor_scale_fp32,
                          block_size: int = NVFP4_BLOCK_SIZE) -> torch.Tensor:
    """Inverse of :func:`quantize_3d_to_nvfp4` (quant.py:188-212): bf16 (E,out,in)."""
    _require_block16(block_size)
    return _nvfp4_dequant(packed_uint8, block_scale_fp8, tensor_scale_fp32)


def dequant_2d_from_nvfp4(packed_uint8, block_scale_fp8, tensor_scale_fp32,
                          block_size: int = NVFP4_BLOCK_SIZE) -> torch.Tensor:
    """Inverse of :func:`quantize_2d_to_nvfp4` (quant.py:233-246)."""
    _require_block16(block_size)
    return _nvfp4_dequant(packed_uint8, block_scale_fp8, tensor_scale_fp32)
