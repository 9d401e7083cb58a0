"""tcgen05 block-scaled GEMM vs the oracle and vs the CUDA-core kernel."""
import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, max_rel_err, randn_bf16, u8
from oracle import gemm as OG

pytestmark = pytest.mark.gpu


@pytest.fixture
def NM():
    from aeo_quant_b200.gpu import nvfp4_matmul
    old = nvfp4_matmul.PATH
    nvfp4_matmul.PATH = "tc"
    yield nvfp4_matmul
    nvfp4_matmul.PATH = old


def _q(x):
    from aeo_quant_b200.gpu import quant as Q
    return Q.quantize_2d_to_nvfp4(x)


@pytest.mark.parametrize("m,n,k", [(128, 1408, 2816), (1, 128, 64), (8, 256, 256), (32, 128, 512),
                                   (64, 2816, 704), (200, 1408, 2816), (256, 384, 1024), (17, 128, 192)])
def test_tc_vs_oracle(NM, m, n, k):
    x = randn_bf16((m, k), 1.0, 1000 + m + k)
    w = randn_bf16((n, k), 0.02, 2000 + n + k)
    ap, asf, ats = _q(x)
    wp, wsf, wts = _q(w)
    wts = wts.float()
    y = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    torch.cuda.synchronize()
    from aeo_quant_b200 import _capi as A
    assert int(A.err_word(y.device).item()) == 0
    ref = OG.nvfp4_gemm(u8(ap), u8(asf), float(ats), u8(wp), u8(wsf), float(wts))
    err = max_rel_err(bf16_to_np(y), ref)
    assert err <= TOL, err


def test_tc_gather_per_slot(NM):
    from aeo_quant_b200.gpu import quant as Q
    E, N, K, m, ksel = 8, 256, 512, 24, 3
    wp, wsf, wts = Q.quantize_3d_to_nvfp4(randn_bf16((E, N, K), 0.02, 3000))
    a = randn_bf16((ksel * m, K), 1.0, 3001)
    ap, asf, ats = _q(a)
    a3p, a3s = ap.reshape(ksel, m, -1), asf.reshape(ksel, m, -1)
    ids = torch.tensor([5, 0, 5], dtype=torch.int64, device="cuda")
    y = NM.nvfp4_linear_3d_gather(a3p, a3s, ats, wp, wsf, wts.float(), ids)
    ref = OG.nvfp4_gemm_3d(u8(a3p), u8(a3s), float(ats), u8(wp), u8(wsf), float(wts), ids.cpu().numpy())
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_tc_matches_simt_bitwise_mostly(NM):
    """Both kernels round once from fp32 sums of exact block products; only the
    summation order differs, so nearly every bf16 output is identical."""
    x = randn_bf16((64, 2816), 1.0, 4000)
    w = randn_bf16((1408, 2816), 0.02, 4001)
    ap, asf, ats = _q(x)
    wp, wsf, wts = _q(w)
    y_tc = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts.float())
    NM.PATH = "simt"
    y_simt = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts.float())
    NM.PATH = "tc"
    same = (y_tc == y_simt).float().mean().item()
    assert same > 0.97, same


def test_weight_atom_cache_follows_the_tensor(NM):
    """A weight allocated where a freed one lived must not reuse its atoms."""
    from aeo_quant_b200.gpu import quant as Q
    x = randn_bf16((16, 512), 1.0, 5000)
    ap, asf, ats = _q(x)
    for seed in (5001, 5002, 5003):
        wp, wsf, wts = _q(randn_bf16((256, 512), 0.02 * (seed - 5000), seed))
        y = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts.float())
        ref = OG.nvfp4_gemm(u8(ap), u8(asf), float(ats), u8(wp), u8(wsf), float(wts))
        assert max_rel_err(bf16_to_np(y), ref) == 0.0
        del wp, wsf, wts, y
