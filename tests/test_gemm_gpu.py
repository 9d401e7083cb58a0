"""Block-scaled NVFP4 GEMMs on the GPU vs the oracle (tolerance TOL)."""
import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, max_rel_err, randn_bf16, u8
from oracle import gemm as OG

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def M():
    from aeo_quant_b200.gpu import nvfp4_matmul, quant
    return nvfp4_matmul, quant


def _q(Q, x):
    return Q.quantize_2d_to_nvfp4(x)


@pytest.mark.parametrize("m,n,k", [(128, 1408, 2816), (1, 1408, 2816), (5, 2816, 704), (64, 256, 128),
                                   (17, 128, 64)])
def test_prequantized_vs_oracle(M, m, n, k):
    NM, Q = M
    x = randn_bf16((m, k), 1.0, 10 + m)
    w = randn_bf16((n, k), 0.02, 20 + n)
    ap, asf, ats = _q(Q, x)
    wp, wsf, wts = _q(Q, w)
    wts = wts.float()                        # checkpoint scale_2 is fp32
    y = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    ref = OG.nvfp4_gemm(u8(ap), u8(asf), float(ats), u8(wp), u8(wsf), float(wts))
    assert max_rel_err(bf16_to_np(y), ref) <= TOL
    yf = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts, out_dtype=torch.float32)
    assert yf.dtype == torch.float32
    ref32 = OG.nvfp4_gemm(u8(ap), u8(asf), float(ats), u8(wp), u8(wsf), float(wts), out="f32")
    assert max_rel_err(yf.cpu().numpy(), ref32) <= 1e-5


def test_linear_flattens_and_requantizes(M):
    NM, Q = M
    x = randn_bf16((2, 3, 704), 1.0, 30)
    w = randn_bf16((256, 704), 0.02, 31)
    wp, wsf, wts = _q(Q, w)
    y = NM.nvfp4_linear(x, wp, wsf, wts.float())
    assert y.shape == (2, 3, 256)
    ref = OG.nvfp4_linear(bf16_to_np(x).reshape(6, 704), u8(wp), u8(wsf), float(wts))
    assert max_rel_err(bf16_to_np(y).reshape(6, 256), ref) <= TOL


@pytest.mark.parametrize("shared", [True, False])
def test_3d_and_gather(M, shared):
    NM, Q = M
    E, N, K, m, ksel = 16, 256, 512, 3, 5
    w = randn_bf16((E, N, K), 0.02, 40)
    wp, wsf, wts = Q.quantize_3d_to_nvfp4(w)
    wts = wts.float()
    if shared:
        a = randn_bf16((m, K), 1.0, 41)
        ap, asf, ats = _q(Q, a)
        a3p, a3s = ap, asf
    else:
        a = randn_bf16((ksel * m, K), 1.0, 42)
        ap, asf, ats = _q(Q, a)
        a3p, a3s = ap.reshape(ksel, m, -1), asf.reshape(ksel, m, -1)
    ids = torch.tensor([7, 0, 15, 7, 3], dtype=torch.int64, device="cuda")
    y = NM.nvfp4_linear_3d_gather(a3p, a3s, ats, wp, wsf, wts, ids)
    assert y.shape == (ksel, m, N)
    ref = OG.nvfp4_gemm_3d(u8(a3p), u8(a3s), float(ats), u8(wp), u8(wsf), float(wts), ids.cpu().numpy())
    assert max_rel_err(bf16_to_np(y), ref) <= TOL
    y32 = NM.nvfp4_linear_3d_gather(a3p, a3s, ats, wp, wsf, wts, ids.to(torch.int32))
    assert torch.equal(y, y32)
    if not shared:
        return
    y3 = NM.nvfp4_linear_3d_prequantized(a3p, a3s, ats, wp, wsf, wts)
    assert y3.shape == (E, m, N)
    ref3 = OG.nvfp4_gemm_3d(u8(a3p), u8(a3s), float(ats), u8(wp), u8(wsf), float(wts))
    assert max_rel_err(bf16_to_np(y3), ref3) <= TOL


def test_bit_stable_across_calls(M):
    NM, Q = M
    x = randn_bf16((4, 2816), 1.0, 50)
    w = randn_bf16((1408, 2816), 0.02, 51)
    ap, asf, ats = _q(Q, x)
    wp, wsf, wts = _q(Q, w)
    y1 = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    y2 = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    assert torch.equal(y1, y2)
