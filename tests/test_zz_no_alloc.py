"""The allocation-free decode entry point, called through the C ABI.

It serves callers that cannot allocate device memory where they run the
expert forward (a serving runtime that reserves all device memory up front,
a plugin without access to its host's allocator). Its output must match the
workspace-taking entry point on the same inputs, on consecutive calls (the
static scratch keeps the previous call's contents). This file is collected
last so a failure here cannot hide any other test's result.
"""
import numpy as np
import pytest
import torch

from helpers import bf16_to_np, randn_bf16, routing

pytestmark = pytest.mark.gpu


def test_noalloc_decode_matches_workspace_entry_point():
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.gpu import quant as Q
    lib = A.load()
    E, H, I, k = 16, 2816, 704, 8
    assert lib.aeoq_moe_nvfp4_decode_fused_supported(k, H, I)
    assert lib.aeoq_moe_nvfp4_decode_fused_workspace_size(k, H, I) <= \
        lib.aeoq_moe_nvfp4_decode_fused_noalloc_max_scratch()
    gp, gs, gt = Q.quantize_3d_to_nvfp4(randn_bf16((E, 2 * I, H), 0.02, 900))
    dp, ds, dt = Q.quantize_3d_to_nvfp4(randn_bf16((E, H, I), 0.02, 901))
    gt, dt = gt.float(), dt.float()
    st = torch.cuda.current_stream().cuda_stream
    ws_n = lib.aeoq_moe_nvfp4_decode_fused_workspace_size(k, H, I)
    ws = torch.zeros(ws_n, dtype=torch.uint8, device="cuda")

    def common(h, idx, w, out):
        return (h.data_ptr(), idx.data_ptr(), A.I64, w.data_ptr(), k, gp.data_ptr(), gs.data_ptr(),
                gt.data_ptr(), A.F32, dp.data_ptr(), ds.data_ptr(), dt.data_ptr(), A.F32, E, H, I,
                out.data_ptr())

    for call in range(2):   # two calls in a row: the static scratch is reused
        h = randn_bf16((1, H), 1.0, 910 + call)
        idx, w = routing(1, E, k, 920 + call)
        idx, w = idx.cuda(), w.cuda()
        ref = torch.empty(1, H, dtype=torch.bfloat16, device="cuda")
        got = torch.full((1, H), float("nan"), dtype=torch.bfloat16, device="cuda")
        A.check(lib.aeoq_moe_nvfp4_decode_fused(*common(h, idx, w, ref), ws.data_ptr(), ws_n, st))
        A.check(lib.aeoq_moe_nvfp4_decode_fused_noalloc(*common(h, idx, w, got), st))
        torch.cuda.synchronize()
        assert np.all(np.isfinite(bf16_to_np(got)))
        # the same kernel on the same inputs: identical bits, so a stale
        # value left in the shared scratch by the previous call would show
        assert torch.equal(got, ref)


def test_noalloc_rejects_oversized_shape():
    from aeo_quant_b200 import _capi as A
    lib = A.load()
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    rc = lib.aeoq_moe_nvfp4_decode_fused_noalloc(p, p, A.I64, p, 16, p, p, p, A.F32, p, p, p, A.F32,
                                                 128, 4096, 2048 * 8, p, 0)
    assert rc != 0
