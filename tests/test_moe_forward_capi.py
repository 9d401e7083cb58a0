"""The whole-layer C entry points (aeoq_moe_nvfp4_forward,
aeoq_moe_fp8_forward), called through ctypes with one workspace, against the
Python layer's launch sequence on the same inputs: the outputs must be
identical bit for bit (same kernels, same order). The Python layer itself is
checked against the oracle in test_moe_gpu.py and test_fp8_gpu.py."""
import pytest
import torch

from helpers import randn_bf16, routing

pytestmark = pytest.mark.gpu

E, H, I, K = 16, 512, 256, 8


@pytest.fixture(scope="module")
def layer():
    from aeo_quant_b200.gpu import quant as Q
    gu = randn_bf16((E, 2 * I, H), 0.02, 31)
    dw = randn_bf16((E, H, I), 0.02, 32)
    nv = Q.quantize_3d_to_nvfp4(gu) + Q.quantize_3d_to_nvfp4(dw)
    f8 = Q.quantize_3d_to_fp8(gu) + Q.quantize_3d_to_fp8(dw)
    return nv, f8


def _inputs(T, seed, drop=False):
    ids, w = routing(T, E, K, seed)
    ids = ids.cuda()
    if drop and T > 2:
        ids[2, 1] = E                      # dropped pair (id == E)
    return randn_bf16((T, H), 1.0, seed + 1), ids, w.to(torch.bfloat16).cuda()


@pytest.mark.parametrize("T,one_token", [(1, True), (1, False), (37, False), (300, False), (64, True)])
def test_nvfp4_forward_matches_python_layer(layer, T, one_token):
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    lib = A.load()
    gp, gs, gt, dp, ds, dt = layer[0]
    x, ids, w = _inputs(T, 40 + T, drop=True)
    ref = moe_ops.nvfp4_experts_grouped(x, ids, w, gp, gs, gt, dp, ds, dt, one_token_semantics=one_token)
    gu_atoms = A.weight_atoms(gs, E, 2 * I, H, geglu_inter=I)
    dw_atoms = A.weight_atoms(ds, E, H, I)
    n = lib.aeoq_moe_nvfp4_forward_workspace_size(T, K, E, H, I)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):                     # the workspace's contents from the first call do not matter
        ws = torch.full((n,), 0xA5, dtype=torch.uint8, device="cuda")
        A.check(lib.aeoq_moe_nvfp4_forward(
            x.data_ptr(), T, ids.data_ptr(), A.dtype_code(ids.dtype), w.data_ptr(), K, gp.data_ptr(),
            gu_atoms.data_ptr(), gt.data_ptr(), A.dtype_code(gt.dtype), dp.data_ptr(), dw_atoms.data_ptr(),
            dt.data_ptr(), A.dtype_code(dt.dtype), E, H, I, 1 if one_token else 0, out.data_ptr(), ws.data_ptr(), n,
            A.err_word(x.device).data_ptr(), A.stream_ptr(x.device)))
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert int(A.err_word(x.device).item()) == 0


@pytest.mark.parametrize("T", [1, 37, 300])
def test_fp8_forward_matches_python_layer(layer, T):
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    lib = A.load()
    gq, gsc, dq, dsc = layer[1]
    gsb = gsc.reshape(-1).float().contiguous()
    dsb = dsc.reshape(-1).float().contiguous()
    x, ids, w = _inputs(T, 60 + T, drop=True)
    ref = moe_ops.fp8_experts_grouped(x, ids, w, gq, gsb, dq, dsb)
    n = lib.aeoq_moe_fp8_forward_workspace_size(T, K, E, H, I)
    ws = torch.full((n,), 0x5A, dtype=torch.uint8, device="cuda")
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    A.check(lib.aeoq_moe_fp8_forward(
        x.data_ptr(), T, ids.data_ptr(), A.dtype_code(ids.dtype), w.data_ptr(), K, gq.view(torch.uint8).data_ptr(),
        gsb.data_ptr(), dq.view(torch.uint8).data_ptr(), dsb.data_ptr(), E, H, I, out.data_ptr(), ws.data_ptr(), n,
        A.err_word(x.device).data_ptr(), A.stream_ptr(x.device)))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_workspace_too_small(layer):
    from aeo_quant_b200 import _capi as A
    lib = A.load()
    gq, gsc, dq, dsc = layer[1]
    x, ids, w = _inputs(5, 70)
    n = lib.aeoq_moe_fp8_forward_workspace_size(5, K, E, H, I)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    out = torch.empty(5, H, dtype=torch.bfloat16, device="cuda")
    rc = lib.aeoq_moe_fp8_forward(x.data_ptr(), 5, ids.data_ptr(), A.dtype_code(ids.dtype), w.data_ptr(), K,
                                  gq.data_ptr(), gsc.data_ptr(), dq.data_ptr(), dsc.data_ptr(), E, H, I,
                                  out.data_ptr(), ws.data_ptr(), n - 1, A.err_word(x.device).data_ptr(),
                                  A.stream_ptr(x.device))
    assert rc == -3 and b"workspace" in lib.aeoq_last_error()
