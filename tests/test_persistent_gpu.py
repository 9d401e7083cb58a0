"""The persistent tensor-core GEMM (224-token tiles for plain GEMMs, 128 for
the grouped expert GEMMs; accumulator double-buffered in TMEM) against the
oracle, at shapes small enough for the CPU oracle."""
import types

import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, max_rel_err, randn_bf16, routing, u8, within_tol_or_ulp
from oracle import gemm as OG
from oracle import moe as OM
from oracle import quant as OQ
from oracle.gemm import fp8_scaled_mm

pytestmark = pytest.mark.gpu


@pytest.fixture
def NM224():
    from aeo_quant_b200.gpu import nvfp4_matmul
    old_path, old_tile = nvfp4_matmul.PATH, nvfp4_matmul.FORCE_TILE_N
    nvfp4_matmul.PATH, nvfp4_matmul.FORCE_TILE_N = "tc", 224
    yield nvfp4_matmul
    nvfp4_matmul.PATH, nvfp4_matmul.FORCE_TILE_N = old_path, old_tile


def _q(x):
    from aeo_quant_b200.gpu import quant as Q
    return Q.quantize_2d_to_nvfp4(x)


@pytest.mark.parametrize("m,n,k", [(224, 128, 256), (1000, 384, 512), (2300, 1408, 704), (37, 256, 192)])
def test_persistent_nvfp4_gemm(NM224, m, n, k):
    x = randn_bf16((m, k), 1.0, 7000 + m)
    w = randn_bf16((n, k), 0.02, 7100 + n)
    ap, asf, ats = _q(x)
    wp, wsf, wts = _q(w)
    y = NM224.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts.float())
    ref = OG.nvfp4_gemm(u8(ap), u8(asf), float(ats), u8(wp), u8(wsf), float(wts))
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_persistent_nvfp4_gather_slots(NM224):
    from aeo_quant_b200.gpu import quant as Q
    E, N, K, m, ksel = 6, 256, 512, 300, 3
    wp, wsf, wts = Q.quantize_3d_to_nvfp4(randn_bf16((E, N, K), 0.02, 7200))
    a = randn_bf16((ksel * m, K), 1.0, 7201)
    ap, asf, ats = _q(a)
    a3p, a3s = ap.reshape(ksel, m, -1), asf.reshape(ksel, m, -1)
    ids = torch.tensor([4, 0, 4], dtype=torch.int64, device="cuda")
    y = NM224.nvfp4_linear_3d_gather(a3p, a3s, ats, wp, wsf, wts.float(), ids)
    ref = OG.nvfp4_gemm_3d(u8(a3p), u8(a3s), float(ats), u8(wp), u8(wsf), float(wts), ids.cpu().numpy())
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_persistent_fp8_gemm():
    """N = 2816 and M = 3136 select the 224-token persistent tiles."""
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.bridges.gemma4.moe_ops import fp8_linear
    from aeo_quant_b200.gpu import quant as Q
    M, N, K = 3136, 2816, 128
    assert A.load().aeoq_nvfp4_tile_n(M, N, 1) == 224
    x = randn_bf16((M, K), 1.0, 7300)
    wq, ws = Q.quantize_2d_to_fp8(randn_bf16((N, K), 0.02, 7301))
    sb = ws.reshape(1, N).float()
    y = fp8_linear(x, wq, sb)
    qx, sx = OQ.quantize_fp8_activation_rows(bf16_to_np(x))
    ref = fp8_scaled_mm(qx, sx, u8(wq.view(torch.uint8)), sb.cpu().numpy())
    assert within_tol_or_ulp(bf16_to_np(y), ref)


def _small_layer(E, H, I, seed):
    from aeo_quant_b200.gpu import quant as Q
    gp, gs, gt = Q.quantize_3d_to_nvfp4(randn_bf16((E, 2 * I, H), 0.02, seed))
    dp, ds, dt = Q.quantize_3d_to_nvfp4(randn_bf16((E, H, I), 0.02, seed + 1))
    return gp, gs, gt.float(), dp, ds, dt.float()


def test_persistent_grouped_nvfp4_experts():
    """~128 rows per expert: the grouped GEMMs take 128-token persistent tiles."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    E, H, I, T, k = 16, 512, 256, 1024, 2
    assert moe_ops.pick_tile_n(T * k, E) == 128
    gp, gs, gt, dp, ds, dt = _small_layer(E, H, I, 7400)
    h = randn_bf16((T, H), 1.0, 7402)
    idx, w = routing(T, E, k, 7403)
    y = moe_ops.nvfp4_experts_grouped(h, idx.cuda(), w.cuda(), gp, gs, gt, dp, ds, dt)
    m = OM.NVFP4Experts(u8(gp), u8(gs), float(gt), u8(dp), u8(ds), float(dt))
    ref = OM.nvfp4_prefill(m, bf16_to_np(h), idx.numpy(), bf16_to_np(w))
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_persistent_grouped_fp8_experts():
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    from aeo_quant_b200.gpu import quant as Q
    E, H, I, T, k = 16, 512, 256, 1024, 2
    gq, gs = Q.quantize_3d_to_fp8(randn_bf16((E, 2 * I, H), 0.02, 7500))
    dq, ds = Q.quantize_3d_to_fp8(randn_bf16((E, H, I), 0.02, 7501))
    h = randn_bf16((T, H), 1.0, 7502)
    idx, w = routing(T, E, k, 7503)
    y = moe_ops.fp8_experts_grouped(h, idx.cuda(), w.cuda(), gq, gs.reshape(-1).float(), dq, ds.reshape(-1).float())
    om = OM.FP8Experts(u8(gq.view(torch.uint8)), gs.float().cpu().numpy().reshape(E, 1, -1),
                       u8(dq.view(torch.uint8)), ds.float().cpu().numpy().reshape(E, 1, -1))
    ref = OM.fp8_experts_forward(om, bf16_to_np(h), idx.numpy(), bf16_to_np(w))
    assert max_rel_err(bf16_to_np(y), ref) <= 1e-2   # composed FP8 forward, as in test_fp8_gpu.py
