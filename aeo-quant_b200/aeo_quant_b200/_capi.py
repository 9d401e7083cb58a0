"""ctypes binding of the sm_100a C-ABI library ``libaeoq_b200.so``.

The library is built in-tree by ``aeo-quant_b200/build.py`` (or
``__graft_entry__.build()``). There is no fallback: if the library is
missing, or the process has no sm_100 GPU, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libaeoq_b200.so")

BF16, F16, F32, I32, I64 = 0, 1, 2, 3, 4
FP8_WEIGHT, FP8_ACTIVATION = 0, 1

_DT = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32, torch.int32: I32,
       torch.int64: I64}

_P, _I, _L, _Z, _F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float

# name -> argtypes (every entry point returns int status unless listed in _RESTYPE)
_SIGS = {
    "aeoq_version": [],
    "aeoq_last_error": [],
    "aeoq_nvfp4_quantize_workspace_size": [_L, _L],
    "aeoq_nvfp4_quantize": [_P, _I, _L, _L, _L, _P, _P, _P, _P, _Z, _P],
    "aeoq_nvfp4_quantize_with_scale": [_P, _I, _L, _L, _L, _P, _P, _P, _P],
    "aeoq_nvfp4_dequantize": [_P, _P, _P, _I, _L, _L, _P, _P],
    "aeoq_fp8_quantize_rows": [_P, _I, _L, _L, _L, _P, _L, _P, _I, _P],
    "aeoq_nvfp4_gemm": [_P, _P, _P, _I, _L, _L, _L, _L,
                        _P, _P, _P, _I, _L, _L, _L, _L,
                        _P, _I, _L, _L, _L, _L, _L, _P, _I, _L, _L, _P],
    "aeoq_moe_nvfp4_decode_workspace_size": [_L, _L, _L],
    "aeoq_moe_nvfp4_decode": [_P, _P, _I, _P, _L, _P, _P, _P, _I, _P, _P, _P, _I, _L, _L, _L,
                              _P, _P, _Z, _P],
}
_SIGS["aeoq_moe_nvfp4_decode_gate_up"] = _SIGS["aeoq_moe_nvfp4_decode"]
_SIGS["aeoq_moe_nvfp4_decode_down"] = _SIGS["aeoq_moe_nvfp4_decode"]
_SIGS["aeoq_moe_nvfp4_decode_fused"] = _SIGS["aeoq_moe_nvfp4_decode"]
_SIGS["aeoq_moe_nvfp4_decode_fused_supported"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_fused_workspace_size"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch"] = []
_SIGS["aeoq_nvfp4_gemm_grouped"] = [_P, _P, _L, _P, _P, _I, _P, _P, _L, _L, _L, _I, _P, _I, _P, _I, _P, _P,
                                     _P, _P, _L, _P, _P]
_SIGS["aeoq_moe_route"] = [_P, _I, _P, _L, _L, _L, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P]
_SIGS["aeoq_gather_rows"] = [_P, _P, _P, _P, _P, _P, _I, _P, _L, _L, _L, _P, _P, _P]
_SIGS["aeoq_requant_rows"] = [_P, _L, _P, _P, _P, _I, _P, _L, _P, _L, _I, _P, _P, _P, _P]
_SIGS["aeoq_selftest_div_rn"] = [_I, _P, _P, _P]
_SIGS["aeoq_fp8_gemm"] = [_P, _P, _L, _P, _P, _L, _L, _P, _P, _P]
_SIGS["aeoq_fp8_gemm_grouped"] = [_P, _P, _L, _P, _P, _I, _P, _P, _L, _L, _L, _I, _P, _P, _L, _P, _P]
_SIGS["aeoq_fp8_quantize_rows_gather"] = [_P, _L, _P, _P, _L, _L, _P, _L, _P, _P]
_SIGS["aeoq_gemma4_router"] = [_P, _L, _P, _P, _P, _L, _L, _L, _L, _F, _F, _P, _P, _P, _P]
_SIGS["aeoq_moe_nvfp4_forward_workspace_size"] = [_L, _L, _L, _L, _L]
_SIGS["aeoq_moe_nvfp4_forward"] = [_P, _L, _P, _I, _P, _L, _P, _P, _P, _I, _P, _P, _P, _I, _L, _L, _L, _I, _P, _P,
                                   _Z, _P, _P]
_SIGS["aeoq_moe_fp8_forward_workspace_size"] = [_L, _L, _L, _L, _L]
_SIGS["aeoq_moe_fp8_forward"] = [_P, _L, _P, _I, _P, _L, _P, _P, _P, _P, _L, _L, _L, _P, _P, _Z, _P, _P]
_SIGS["aeoq_moe_nvfp4_decode_tc_supported"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_tc_workspace_size"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_tc"] = [_P, _P, _I, _P, _L, _P, _P, _P, _I, _P, _P, _P, _I, _L, _L, _L, _P, _P, _Z, _P, _P]
_SIGS["aeoq_moe_nvfp4_decode_stream_supported"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_stream_workspace_size"] = [_L, _L, _L]
_SIGS["aeoq_moe_nvfp4_decode_stream"] = _SIGS["aeoq_moe_nvfp4_decode_tc"]
_SIGS["aeoq_nvfp4_tile_n"] = [_L, _L, _L]
_SIGS["aeoq_nvfp4_weight_atoms_size"] = [_L, _L]
_SIGS["aeoq_nvfp4_act_atoms_size"] = [_L, _L, _I]
_SIGS["aeoq_nvfp4_sf_to_atoms"] = [_P, _L, _L, _L, _L, _P, _P]
_SIGS["aeoq_nvfp4_rows_to_tile_atoms"] = [_P, _L, _L, _L, _I, _P, _P]
_SIGS["aeoq_moe_combine"] = [_P, _P, _P, _I, _L, _L, _L, _I, _P, _P]
_SIGS["aeoq_nvfp4_gemm_tc"] = [_P, _P, _P, _I, _L, _P, _P, _P, _I, _L, _P, _I, _L, _L, _L, _L, _I, _P, _I, _P, _P]
_SIGS["aeoq_moe_nvfp4_decode_fused_noalloc"] = [_P, _P, _I, _P, _L, _P, _P, _P, _I, _P, _P, _P, _I, _L, _L, _L,
                                                _P, _P]
_SIGS["aeoq_ep_nccl_unique_id_bytes"] = []
_SIGS["aeoq_ep_nccl_unique_id"] = [_P, _Z]
_SIGS["aeoq_ep_nccl_comm_init"] = [_P, _I, _I, _P]
_SIGS["aeoq_ep_nccl_comm_destroy"] = [_P]
_SIGS["aeoq_ep_dispatch_workspace_size"] = [_I, _L, _L, _L]
_SIGS["aeoq_ep_dispatch"] = [_P, _I, _I, _P, _L, _L, _P, _I, _P, _L, _L, _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]
_SIGS["aeoq_ep_experts_nvfp4_workspace_size"] = [_L, _L, _L, _L, _L, _L]
_SIGS["aeoq_ep_experts_nvfp4"] = [_P, _P, _P, _L, _P, _P, _L, _L, _P, _P, _P, _I, _P, _P, _P, _I, _L, _L, _L, _P, _P,
                                  _Z, _P, _P]
_SIGS["aeoq_ep_combine_workspace_size"] = [_I, _L, _L]
_SIGS["aeoq_ep_combine"] = [_P, _I, _I, _P, _P, _L, _L, _P, _P, _Z, _P]
_RESTYPE = {"aeoq_moe_nvfp4_decode_tc_workspace_size": C.c_size_t,
            "aeoq_ep_nccl_unique_id_bytes": C.c_size_t, "aeoq_ep_dispatch_workspace_size": C.c_size_t,
            "aeoq_ep_experts_nvfp4_workspace_size": C.c_size_t, "aeoq_ep_combine_workspace_size": C.c_size_t,
            "aeoq_moe_nvfp4_decode_stream_workspace_size": C.c_size_t,
            "aeoq_nvfp4_weight_atoms_size": C.c_size_t, "aeoq_nvfp4_act_atoms_size": C.c_size_t,
            "aeoq_last_error": C.c_char_p, "aeoq_nvfp4_quantize_workspace_size": C.c_size_t,
            "aeoq_moe_nvfp4_decode_workspace_size": C.c_size_t,
            "aeoq_moe_nvfp4_decode_fused_workspace_size": C.c_size_t,
            "aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch": C.c_size_t,
            "aeoq_moe_nvfp4_forward_workspace_size": C.c_size_t,
            "aeoq_moe_fp8_forward_workspace_size": C.c_size_t}

_lib = None


class AeoqError(RuntimeError):
    pass


def lib_path() -> str:
    return _LIB_PATH


def load():
    """Load the library (once) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise AeoqError(f"aeo_quant_b200 native library not built: {_LIB_PATH} is missing "
                        "(run aeo-quant_b200/build.py)")
    lib = C.CDLL(_LIB_PATH)
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, C.c_int)
    _lib = lib
    return lib


def exported_symbols():
    return list(_SIGS)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def check(rc: int) -> None:
    if rc != 0:
        msg = load().aeoq_last_error().decode(errors="replace")
        if rc == -1:
            raise ValueError(msg)
        raise AeoqError(f"aeoq status {rc}: {msg}")


_SM100_DEVICES: set = set()


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise AeoqError("aeo_quant_b200 runs on CUDA tensors only (no CPU path); "
                            f"got a tensor on {t.device}")
    dev = tensors[0].device
    if dev.index in _SM100_DEVICES:
        return
    major, _ = torch.cuda.get_device_capability(dev)
    if major != 10:
        raise AeoqError(f"aeo_quant_b200 is built for sm_100a (B200); device {dev} is sm_{major}x")
    _SM100_DEVICES.add(dev.index)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_ERR_WORDS: dict = {}


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 that the tensor-core kernels' bounded waits set on a stall."""
    key = device.index
    t = _ERR_WORDS.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR_WORDS[key] = t
    return t


# Weight scale atoms are derived once per weight tensor and cached here,
# keyed on the tensor's storage, shape and version counter (an in-place
# update of the scales invalidates the entry). Each entry also holds a weak
# reference to the tensor it was built from: memory freed and reused by a
# new tensor at the same address finds a dead reference and rebuilds.
_ATOMS: dict = {}
_ATOMS_MAX = 256


def weight_atoms(sf: torch.Tensor, groups: int, rows_per_group: int, K: int, geglu_inter: int = 0) -> torch.Tensor:
    import weakref
    key = (sf.data_ptr(), tuple(sf.shape), tuple(sf.stride()), sf._version, groups, rows_per_group, K, geglu_inter)
    hit = _ATOMS.get(key)
    if hit is not None:
        ref, t = hit
        if ref() is sf:
            return t
        del _ATOMS[key]
    src = sf
    lib = load()
    sf = sf.contiguous()
    n = lib.aeoq_nvfp4_weight_atoms_size(groups * rows_per_group, K)
    t = torch.empty(max(n, 16), dtype=torch.uint8, device=sf.device)
    check(lib.aeoq_nvfp4_sf_to_atoms(sf.data_ptr(), groups, rows_per_group, K, geglu_inter, t.data_ptr(),
                                     stream_ptr(sf.device)))
    if len(_ATOMS) >= _ATOMS_MAX:
        _ATOMS.pop(next(iter(_ATOMS)))
    _ATOMS[key] = (weakref.ref(src), t)
    return t
