"""Block-scaled NVFP4 matmul on B200 — drop-in for ``aeo_quant.gpu.nvfp4_matmul``.

Same public functions, argument meaning, output shapes and ``ValueError``
conditions as aeo_quant ``src/aeo_quant/gpu/nvfp4_matmul.py``:

* :func:`nvfp4_linear` (:357-396) — quantize activation, then GEMM;
* :func:`nvfp4_linear_prequantized` (:399-519) — 2D GEMM;
* :func:`nvfp4_linear_3d_prequantized` (:522-686) — batched per expert;
* :func:`nvfp4_linear_3d_gather` (:689-864) — batched with in-kernel expert
  gather through ``expert_ids``.

Math: ``C = out(alpha * sum_k (a_k sA)(w_k sW))`` with ``alpha =
f32(a_ts) * f32(w_ts)`` read on the device (no host sync; graph capturable).
The packed bytes are consumed in the reference layout (high nibble = even k).
Unlike the Triton launchers no zero-padding copies are made: the kernels
bound M themselves.
"""
from __future__ import annotations

import torch

from .. import _capi as A
from .quant import quantize_2d_to_nvfp4

FP8_E4M3_MAX = 448.0
FP4_E2M1_MAX = 6.0
NVFP4_BLOCK_SIZE = 16

_OUT_DT = {torch.bfloat16: A.BF16, torch.float32: A.F32}


def _quantize_bf16_activation_to_nvfp4(x_bf16: torch.Tensor):
    """Activation quant used by :func:`nvfp4_linear` (nvfp4_matmul.py:338-354):
    global tensor scale plus per-16 block scales, as ``quantize_2d_to_nvfp4``."""
    return quantize_2d_to_nvfp4(x_bf16)


def _check_nk(N: int, K: int, pad_msg: str) -> None:
    # Same divisibility contract as the reference launchers (:457-476).
    BLOCK_N = 128
    BLOCK_K = 128 if K % 128 == 0 else 64
    if N % BLOCK_N != 0:
        raise ValueError(f"N={N} must be divisible by BLOCK_N={BLOCK_N}. {pad_msg}")
    if K % BLOCK_K != 0:
        raise ValueError(f"K={K} must be divisible by BLOCK_K={BLOCK_K}. {pad_msg}")


def _out_code(out_dtype: torch.dtype) -> int:
    if out_dtype not in _OUT_DT:
        raise ValueError(f"out_dtype must be torch.bfloat16 or torch.float32, got {out_dtype}")
    return _OUT_DT[out_dtype]


# Which kernel serves a GEMM: "auto" picks the tcgen05 kernel once M reaches
# TC_MIN_M rows (below that the problem is a weight stream that the CUDA-core
# gather GEMV serves), "tc" / "simt" force one (used by the tests).
PATH = "auto"
TC_MIN_M = 8
FORCE_TILE_N = 0   # tests: force the token-tile width of the tensor-core GEMM


def _gemm(a, a_sf, a_ts, w, w_sf, w_ts, ids, slots, M, N, K, a_shared, out_dtype):
    """Launch the block-scaled GEMM. ``a``/``a_sf`` are (M,K/2)/(M,K/16) when
    ``a_shared`` else (slots,M,...); ``w``/``w_sf`` are (E,N,...)."""
    A.require_cuda(a, a_sf, a_ts, w, w_sf, w_ts)
    lib = A.load()
    a = a.contiguous()
    a_sf = a_sf.contiguous()
    w = w.contiguous()
    w_sf = w_sf.contiguous()
    c = torch.empty(slots, M, N, dtype=out_dtype, device=a.device)
    use_tc = PATH == "tc" or (PATH == "auto" and M >= TC_MIN_M)
    if use_tc:
        ids_p, ids_dt = (None, 0) if ids is None else (ids.data_ptr(), A.dtype_code(ids.dtype))
        tile_n = FORCE_TILE_N or lib.aeoq_nvfp4_tile_n(M, N, slots)
        a_rows = M if a_shared else slots * M
        tiles = (M + tile_n - 1) // tile_n * (1 if a_shared else slots)
        a_atoms = torch.empty(max(lib.aeoq_nvfp4_act_atoms_size(tiles, K, tile_n), 16), dtype=torch.uint8,
                              device=a.device)
        A.check(lib.aeoq_nvfp4_rows_to_tile_atoms(a_sf.data_ptr(), a_rows, M, K, tile_n, a_atoms.data_ptr(),
                                                  A.stream_ptr(a.device)))
        w_atoms = A.weight_atoms(w_sf, w.shape[0], N, K)
        A.check(lib.aeoq_nvfp4_gemm_tc(
            a.data_ptr(), a_atoms.data_ptr(), a_ts.data_ptr(), A.dtype_code(a_ts.dtype), 0 if a_shared else M,
            w.data_ptr(), w_atoms.data_ptr(), w_ts.data_ptr(), A.dtype_code(w_ts.dtype), w.shape[0],
            ids_p, ids_dt, slots, M, N, K, tile_n, c.data_ptr(), _out_code(out_dtype),
            A.err_word(a.device).data_ptr(), A.stream_ptr(a.device)))
        return c
    es = c.element_size()
    if a_shared:
        a_ss, a_sfss = 0, 0
    else:
        a_ss, a_sfss = M * (K // 2), M * (K // 16)
    ids_p, ids_dt, n_exp = (None, 0, w.shape[0]) if ids is None else (ids.data_ptr(), A.dtype_code(ids.dtype), w.shape[0])
    A.check(lib.aeoq_nvfp4_gemm(
        a.data_ptr(), a_sf.data_ptr(), a_ts.data_ptr(), A.dtype_code(a_ts.dtype),
        a_ss, K // 2, a_sfss, K // 16,
        w.data_ptr(), w_sf.data_ptr(), w_ts.data_ptr(), A.dtype_code(w_ts.dtype),
        N * (K // 2), K // 2, N * (K // 16), K // 16,
        ids_p, ids_dt, n_exp, slots, M, N, K,
        c.data_ptr(), _out_code(out_dtype), M * N * es, N * es, A.stream_ptr(a.device)))
    return c


def nvfp4_linear(
    x_bf16: torch.Tensor,
    w_packed: torch.Tensor,
    w_block_scale: torch.Tensor,
    w_tensor_scale: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """One expert's NVFP4 matmul: (..., K) bf16 input x (N, K) NVFP4 weight
    (nvfp4_matmul.py:357-396). Returns (..., N) of ``out_dtype``."""
    orig_shape = x_bf16.shape
    if x_bf16.ndim != 2:
        x_bf16 = x_bf16.reshape(-1, orig_shape[-1])
    a_packed, a_block_scale, a_tensor_scale = _quantize_bf16_activation_to_nvfp4(x_bf16)
    out = nvfp4_linear_prequantized(
        a_packed, a_block_scale, a_tensor_scale,
        w_packed, w_block_scale, w_tensor_scale,
        out_dtype=out_dtype,
    )
    if len(orig_shape) > 2:
        out = out.reshape(*orig_shape[:-1], out.shape[-1])
    return out


def nvfp4_linear_prequantized(
    a_packed: torch.Tensor,
    a_block_scale: torch.Tensor,
    a_tensor_scale: torch.Tensor,
    w_packed: torch.Tensor,
    w_block_scale: torch.Tensor,
    w_tensor_scale: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """(M, K/2) prequantized activation x (N, K/2) weight -> (M, N)
    (nvfp4_matmul.py:399-519)."""
    M = a_packed.shape[0]
    K = a_packed.shape[1] * 2
    N = w_packed.shape[0]
    _check_nk(N, K, "Add padding upstream if needed.")
    return _gemm(a_packed, a_block_scale, a_tensor_scale, w_packed.unsqueeze(0),
                 w_block_scale.unsqueeze(0), w_tensor_scale, None, 1, M, N, K, True, out_dtype)[0]


def _canon_activation(a_packed, a_block_scale, n_slots, what):
    if a_packed.ndim == 2:
        M, K_half_a = a_packed.shape
        return a_packed, a_block_scale, M, K_half_a, True
    if a_packed.ndim == 3:
        E_a, M, K_half_a = a_packed.shape
        if E_a != n_slots:
            raise ValueError(what.format(E_a=E_a, n=n_slots))
        return a_packed, a_block_scale, M, K_half_a, False
    raise ValueError(
        f"a_packed must be 2D (shared) or 3D (per-expert); "
        f"got shape {tuple(a_packed.shape)}"
    )


def nvfp4_linear_3d_prequantized(
    a_packed: torch.Tensor,
    a_block_scale: torch.Tensor,
    a_tensor_scale: torch.Tensor,
    w_packed: torch.Tensor,
    w_block_scale: torch.Tensor,
    w_tensor_scale: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """Batched per-expert NVFP4 matmul (nvfp4_matmul.py:522-686).

    ``a_packed`` (M, K/2) is shared by every expert, (E, M, K/2) is per
    expert. Weights (E, N, K/2). Returns (E, M, N).
    """
    if w_packed.ndim != 3:
        raise ValueError(
            f"w_packed must be 3D (E, N, K//2); got shape {tuple(w_packed.shape)}"
        )
    E, N, K_half_w = w_packed.shape
    a_packed, a_block_scale, M, K_half_a, shared = _canon_activation(
        a_packed, a_block_scale, E, "per-expert activation E={E_a} must equal weight E={n}")
    if K_half_a != K_half_w:
        raise ValueError(
            f"activation K//2={K_half_a} must equal weight K//2={K_half_w}"
        )
    K = K_half_a * 2
    _check_nk(N, K, "Pad upstream.")
    return _gemm(a_packed, a_block_scale, a_tensor_scale, w_packed, w_block_scale, w_tensor_scale,
                 None, E, M, N, K, shared, out_dtype)


def nvfp4_linear_3d_gather(
    a_packed: torch.Tensor,
    a_block_scale: torch.Tensor,
    a_tensor_scale: torch.Tensor,
    w_packed: torch.Tensor,
    w_block_scale: torch.Tensor,
    w_tensor_scale: torch.Tensor,
    expert_ids: torch.Tensor,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
) -> torch.Tensor:
    """Batched NVFP4 matmul with in-kernel expert gather (nvfp4_matmul.py:689-864).

    Weights are the full (E_FULL, N, K/2) tensor; slot j reads expert
    ``expert_ids[j]`` (int32 or int64, read on the device). Returns
    (K_SELECTED, M, N).
    """
    if w_packed.ndim != 3:
        raise ValueError(
            f"w_packed must be 3D (E_FULL, N, K//2); "
            f"got shape {tuple(w_packed.shape)}"
        )
    E_full, N, K_half_w = w_packed.shape
    if expert_ids.ndim != 1:
        raise ValueError(
            f"expert_ids must be 1D; got shape {tuple(expert_ids.shape)}"
        )
    K_selected = expert_ids.shape[0]
    if expert_ids.dtype not in (torch.int32, torch.int64):
        expert_ids = expert_ids.to(torch.int32)
    if not expert_ids.is_contiguous():
        expert_ids = expert_ids.contiguous()
    a_packed, a_block_scale, M, K_half_a, shared = _canon_activation(
        a_packed, a_block_scale, K_selected,
        "per-expert activation E={E_a} must equal len(expert_ids)={n}")
    if K_half_a != K_half_w:
        raise ValueError(
            f"activation K//2={K_half_a} must equal weight K//2={K_half_w}"
        )
    K = K_half_a * 2
    _check_nk(N, K, "Pad upstream.")
    return _gemm(a_packed, a_block_scale, a_tensor_scale, w_packed, w_block_scale, w_tensor_scale,
                 expert_ids, K_selected, M, N, K, shared, out_dtype)
