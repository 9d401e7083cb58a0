"""CPU checks of the C-ABI library: it loads, exports every declared symbol,
and rejects bad arguments before touching the GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "aeoq.h")


def declared_symbols():
    with open(HEADER) as f:
        src = f.read()
    return sorted(set(re.findall(r"AEOQ_API\s+[\w\s\*]+?\b(aeoq_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from aeo_quant_b200 import _capi
    return _capi.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "aeoq_nvfp4_quantize" in syms and "aeoq_moe_nvfp4_decode" in syms
    assert len(syms) >= 8


def test_library_exports_every_declared_symbol(lib):
    from aeo_quant_b200 import _capi
    raw = ctypes.CDLL(_capi.lib_path())
    for s in declared_symbols():
        assert hasattr(raw, s), f"{s} declared in include/aeoq.h but not exported"
    # and the ctypes table binds exactly the header
    assert sorted(_capi.exported_symbols()) == declared_symbols()


def test_version_and_error_string(lib):
    assert lib.aeoq_version() >= 100
    assert isinstance(lib.aeoq_last_error(), bytes)


def test_argument_validation_without_gpu(lib):
    # K not a multiple of 16: rejected before any CUDA call
    rc = lib.aeoq_nvfp4_quantize(None, 0, 4, 24, 24, None, None, None, None, 0, None)
    assert rc == -1
    assert b"divisible by block_size" in lib.aeoq_last_error()
    rc = lib.aeoq_nvfp4_quantize(None, 7, 4, 32, 32, None, None, None, None, 0, None)
    assert rc == -1
    rc = lib.aeoq_fp8_quantize_rows(None, 0, 4, 32, 32, None, 32, None, 5, None)
    assert rc == -1 and b"mode" in lib.aeoq_last_error()
    rc = lib.aeoq_moe_nvfp4_decode(None, None, 4, None, 8, None, None, None, 2, None, None, None, 2,
                                   128, 2816, 704, None, None, 0, None)
    assert rc == -1
    rc = lib.aeoq_moe_nvfp4_decode(None, None, 4, None, 99, None, None, None, 2, None, None, None, 2,
                                   128, 2816, 704, None, None, 0, None)
    assert rc == -1 and b"top_k" in lib.aeoq_last_error()


def test_workspace_sizes(lib):
    assert lib.aeoq_nvfp4_quantize_workspace_size(1, 2816) == 0
    assert lib.aeoq_nvfp4_quantize_workspace_size(1408, 2816) > 0
    assert lib.aeoq_moe_nvfp4_decode_workspace_size(8, 2816, 704) >= 8 * 704 * 2
    # whole-layer forwards: at least the sorted (pairs, H) bf16 outputs, growing with T, 0 for no tokens
    for fn in (lib.aeoq_moe_nvfp4_forward_workspace_size, lib.aeoq_moe_fp8_forward_workspace_size):
        assert fn(0, 8, 128, 2816, 704) == 0
        assert fn(64, 8, 128, 2816, 704) >= 64 * 8 * 2816 * 2
        assert fn(4096, 8, 128, 2816, 704) > fn(64, 8, 128, 2816, 704)


def test_whole_layer_forward_validation(lib):
    # no tokens: nothing to do, no pointer touched
    assert lib.aeoq_moe_nvfp4_forward(None, 0, None, 4, None, 8, None, None, None, 2, None, None, None, 2,
                                      128, 2816, 704, 0, None, None, 0, None, None) == 0
    rc = lib.aeoq_moe_nvfp4_forward(None, 4, None, 4, None, 99, None, None, None, 2, None, None, None, 2,
                                    128, 2816, 704, 0, None, None, 0, None, None)
    assert rc == -1 and b"bad shape" in lib.aeoq_last_error()
    rc = lib.aeoq_moe_fp8_forward(None, 4, None, 4, None, 8, None, None, None, None, 128, 2816, 704, None,
                                  None, 0, None, None)
    assert rc == -1 and b"null pointer" in lib.aeoq_last_error()


def test_python_api_refuses_cpu_tensors():
    import torch
    from aeo_quant_b200.gpu import quant as Q
    from aeo_quant_b200 import AeoqError
    with pytest.raises(AeoqError):
        Q.quantize_2d_to_nvfp4(torch.zeros(2, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="expects a 2D tensor"):
        Q.quantize_2d_to_nvfp4(torch.zeros(2, 2, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="must be divisible by block_size"):
        Q.quantize_3d_to_nvfp4(torch.zeros(1, 2, 24, dtype=torch.bfloat16))


def test_matmul_shape_errors_match_reference():
    import torch
    from aeo_quant_b200.gpu import nvfp4_matmul as NM
    a = torch.zeros(4, 64, dtype=torch.uint8)
    s = torch.zeros(4, 8, dtype=torch.uint8)
    t = torch.zeros(())
    with pytest.raises(ValueError, match="must be divisible by BLOCK_N=128"):
        NM.nvfp4_linear_prequantized(a, s, t, torch.zeros(100, 64, dtype=torch.uint8), s, t)
    with pytest.raises(ValueError, match="w_packed must be 3D"):
        NM.nvfp4_linear_3d_gather(a, s, t, torch.zeros(128, 64, dtype=torch.uint8), s, t,
                                  torch.zeros(2, dtype=torch.int64))
    with pytest.raises(ValueError, match="expert_ids must be 1D"):
        NM.nvfp4_linear_3d_gather(a, s, t, torch.zeros(2, 128, 64, dtype=torch.uint8), s, t,
                                  torch.zeros(2, 1, dtype=torch.int64))


def test_expert_parallel_entries_without_gpu(lib):
    """The expert-parallel C entries check their arguments before any NCCL or
    CUDA call, and size their workspaces from the shapes alone."""
    assert lib.aeoq_ep_nccl_unique_id_bytes() == 128
    # no communicator
    rc = lib.aeoq_ep_dispatch(None, 2, 0, None, 48, 2816, None, 4, None, 8, 16, None, None, None, None, None, None,
                              None, None, 0, None)
    assert rc == -1 and b"ep_dispatch" in lib.aeoq_last_error()
    # experts not divisible over the ranks
    rc = lib.aeoq_ep_dispatch(1, 3, 0, None, 48, 2816, None, 4, None, 8, 16, None, None, None, None, None, None,
                              None, None, 0, None)
    assert rc == -1 and b"multiple of world" in lib.aeoq_last_error()
    rc = lib.aeoq_ep_combine(None, 2, 5, None, None, 48, 2816, None, None, 0, None)
    assert rc == -1
    # dispatch: amax + this rank's quantized rows + the per-destination ids
    n = lib.aeoq_ep_dispatch_workspace_size(2, 48, 8, 2816)
    assert n >= 48 * 2816 // 2 + 48 * 2816 // 16 + 2 * 48 * 8 * 4
    assert lib.aeoq_ep_dispatch_workspace_size(2, 0, 8, 2816) == 0
    # combine: the returned rows of every rank
    assert lib.aeoq_ep_combine_workspace_size(2, 48, 2816) >= 2 * 48 * 2816 * 2
    # experts: at least the sorted (pairs, H) bf16 outputs
    assert lib.aeoq_ep_experts_nvfp4_workspace_size(96, 8, 384, 8, 2816, 704) >= 96 * 8 * 2816 * 2
