"""Parity at the sizes bench.py times, against the oracle.

* the single-linear NVFP4 GEMM (N = 1408, K = 2816) at M = 8192 and 32768
  rows, which run the persistent 224-token-tile kernel; the oracle checks a
  seeded sample of output rows (each row depends only on its own activation
  row and the weights);
* the grouped expert forwards at 4096 tokens, top-8 over 128 experts
  (32,768 token-expert pairs), NVFP4 and FP8, against the full oracle;
* one expert-parallel-shaped layer at 8192 tokens with Zipf(1.2)-skewed
  top-8 routing (hot experts with thousands of rows), NVFP4, full oracle.

The FP8 forward re-quantizes each GeGLU row to e4m3. A gate_up output one
bf16 ulp from the f64 oracle (f32 accumulation order) can move one e4m3
code of that row, which the down projection spreads over the output row.
The test proves that this is the only source of error above the bar: it
feeds the oracle's down projection and combine with the GPU's own gate_up
rows, and requires the GPU output within 2e-3 * max|ref| (or one bf16 ulp)
of that; it requires every GPU gate_up value within one bf16 ulp of the
oracle's (or, for outputs near zero after cancellation, within 1e-4 of the
block's largest), and bounds how many differ at all.
"""
import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, bf16_ulp, max_rel_err, randn_bf16, u8, within_tol_or_ulp
from oracle import gemm as OG
from oracle import moe as OM
from oracle import numerics as N

pytestmark = pytest.mark.gpu

E, H, I, K_TOP = 128, 2816, 704, 8


def softmax_topk_routing(T, seed):
    """top-8 by softmax over N(0,1) logits, weights renormalised (bench.py's routing)."""
    g = torch.Generator().manual_seed(seed)
    p = torch.softmax(torch.randn(T, E, generator=g), -1)
    wv, ids = torch.topk(p, K_TOP, dim=-1)
    return ids, (wv / wv.sum(-1, keepdim=True)).to(torch.bfloat16)


def zipf_routing(T, seed, s=1.2):
    """Eight distinct experts per token drawn from Zipf(s) over a seeded expert permutation."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(E, generator=g)
    p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** s
    ids = perm[torch.multinomial(p.expand(T, E), K_TOP, replacement=False, generator=g)]
    w = torch.softmax(torch.randn(T, K_TOP, generator=g), -1).to(torch.bfloat16)
    return ids, w


@pytest.mark.parametrize("M", [8192, 32768])
def test_persistent_gemm_benched_rows(M):
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.gpu import nvfp4_matmul as NM
    from aeo_quant_b200.gpu import quant as Q
    Nw, K = 1408, 2816
    assert A.load().aeoq_nvfp4_tile_n(M, Nw, 1) == 224
    wp, wsf, wts = Q.quantize_2d_to_nvfp4(randn_bf16((Nw, K), 0.02, 8000))
    x = randn_bf16((M, K), 1.0, 8001 + M)
    ap, asf, ats = Q.quantize_2d_to_nvfp4(x)
    y = NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts.float())
    rows = np.sort(np.random.default_rng(M).choice(M, 512, replace=False))
    # first and last tiles too (partial-tile and schedule edges)
    rows = np.unique(np.r_[rows, np.arange(224), np.arange(M - 224, M)])
    ri = torch.from_numpy(rows).cuda()
    ref = OG.nvfp4_gemm(u8(ap[ri]), u8(asf[ri]), float(ats), u8(wp), u8(wsf), float(wts))
    assert max_rel_err(bf16_to_np(y[ri]), ref) <= TOL


@pytest.fixture(scope="module")
def nvfp4_layer():
    from aeo_quant_b200.gpu import quant as Q
    gp, gs, gt = Q.quantize_3d_to_nvfp4(randn_bf16((E, 2 * I, H), 0.02, 8100))
    dp, ds, dt = Q.quantize_3d_to_nvfp4(randn_bf16((E, H, I), 0.02, 8101))
    gt, dt = gt.float(), dt.float()
    om = OM.NVFP4Experts(u8(gp), u8(gs), float(gt), u8(dp), u8(ds), float(dt))
    return (gp, gs, gt, dp, ds, dt), om


@pytest.mark.parametrize("T,routing_kind", [(4096, "softmax"), (8192, "zipf")])
def test_nvfp4_grouped_benched_size(nvfp4_layer, T, routing_kind):
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    (gp, gs, gt, dp, ds, dt), om = nvfp4_layer
    h = randn_bf16((T, H), 1.0, 8200 + T)
    ids, w = softmax_topk_routing(T, 8300) if routing_kind == "softmax" else zipf_routing(T, 8301)
    if routing_kind == "zipf":
        assert int(torch.bincount(ids.reshape(-1), minlength=E).max()) > 4096   # hot experts
    y = moe_ops.nvfp4_experts_grouped(h, ids.cuda(), w.cuda(), gp, gs, gt, dp, ds, dt)
    ref = OM.nvfp4_prefill(om, bf16_to_np(h), ids.numpy(), bf16_to_np(w))
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def _fp8_forward_with_gate_up(m, hidden, ids, wts, gate_up_of):
    """``fp8_experts_forward`` (modeling.py:110-146) with each expert's
    gate_up rows taken from ``gate_up_of(e, token_rows)`` instead of the
    oracle GEMM; everything after it is the oracle's."""
    final = np.zeros_like(hidden)
    for e in np.unique(ids):
        pos, tok = np.nonzero(ids.T == e)
        cur = OM.geglu(gate_up_of(e, tok))
        d = OM.fp8_linear(cur, m.down_proj[e], m.down_proj_scale[e])
        d = N.bf16(d * wts[tok, pos][:, None])
        final[tok] = N.bf16(final[tok] + d)
    return final


def test_fp8_grouped_benched_size():
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    from aeo_quant_b200.gpu import quant as Q
    T = 4096
    gq, gs = Q.quantize_3d_to_fp8(randn_bf16((E, 2 * I, H), 0.02, 8400))
    dq, ds = Q.quantize_3d_to_fp8(randn_bf16((E, H, I), 0.02, 8401))
    gsb, dsb = gs.reshape(-1).float().contiguous(), ds.reshape(-1).float().contiguous()
    h = randn_bf16((T, H), 1.0, 8402)
    ids, w = softmax_topk_routing(T, 8403)
    y = bf16_to_np(moe_ops.fp8_experts_grouped(h, ids.cuda(), w.cuda(), gq, gsb, dq, dsb))
    om = OM.FP8Experts(u8(gq.view(torch.uint8)), gs.float().cpu().numpy().reshape(E, 1, -1),
                       u8(dq.view(torch.uint8)), ds.float().cpu().numpy().reshape(E, 1, -1))
    hn, idn, wn = bf16_to_np(h), ids.numpy(), bf16_to_np(w)
    ref = OM.fp8_experts_forward(om, hn, idn, wn)

    # the GPU's gate_up rows of every expert (the same tensor-core GEMM and
    # per-row activation quantization as the grouped forward)
    flips, total = 0, 0

    def gpu_gate_up(e, tok):
        nonlocal flips, total
        rows = h[torch.from_numpy(tok).cuda()]
        gu = bf16_to_np(moe_ops.fp8_linear(rows, gq[e], gs[e].reshape(1, -1).float()))
        gu_ref = OM.fp8_linear(hn[tok], om.gate_up_proj[e], om.gate_up_proj_scale[e])
        diff = np.abs(gu.astype(np.float64) - gu_ref)
        # one bf16 ulp, or (outputs near zero after cancellation) the f32
        # accumulation error of 2816 products, far below 1e-4 * max|ref|
        lim = np.maximum(bf16_ulp(gu_ref), 1e-4 * np.max(np.abs(gu_ref)))
        assert np.all(diff <= lim), ("gate_up beyond one bf16 ulp", float(np.max(diff / lim)))
        flips += int(np.count_nonzero(diff))
        total += gu.size
        return gu

    mixed = _fp8_forward_with_gate_up(om, hn, idn, wn, gpu_gate_up)
    # every output within the bar of the oracle fed with the GPU's gate_up rows
    assert within_tol_or_ulp(y, mixed)
    # one-ulp gate_up flips are rare (f32 accumulation order at a bf16 boundary)
    assert flips <= 1e-3 * total, (flips, total)
    # and against the pure oracle, the rows above the bar are few
    lim = TOL * np.max(np.abs(ref))
    bad_rows = int(np.count_nonzero(np.any(np.abs(y - ref) > np.maximum(lim, bf16_ulp(ref)), axis=1)))
    print(f"fp8 T={T}: gate_up flips {flips}/{total}, token rows above the bar vs pure oracle {bad_rows}/{T}, "
          f"max rel err {max_rel_err(y, ref):.2e}")
    assert bad_rows <= max(8, T // 64)
