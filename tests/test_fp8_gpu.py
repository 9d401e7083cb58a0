"""FP8 path on the GPU: per-row activation quantization (bit-exact), the
tensor-core FP8 GEMM (tolerance vs the f32 oracle), and
Gemma4TextExpertsFP8.forward vs the reference-generated golden outputs and
the oracle restatement at the Gemma-4 expert shapes."""
import types

import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, bits_to_bf16, max_rel_err, randn_bf16, routing, u8, within_tol_or_ulp
from oracle import moe as OM
from oracle import numerics as N
from oracle import quant as OQ
from oracle.gemm import fp8_scaled_mm

pytestmark = pytest.mark.gpu


def make_fp8_module(E, H, I, gu, gs, dw, ds):
    from aeo_quant_b200.bridges.gemma4.modeling import Gemma4TextExpertsFP8
    cfg = types.SimpleNamespace(num_experts=E, hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")
    m = Gemma4TextExpertsFP8(cfg).cuda()
    m.gate_up_proj.data.copy_(gu)
    m.down_proj.data.copy_(dw)
    # the loader's preconverted layout: (E, 1, N) f32 (loader.py:47-64)
    m.gate_up_proj_scale = gs.reshape(E, 1, 2 * I).float().contiguous()
    m.down_proj_scale = ds.reshape(E, 1, H).float().contiguous()
    return m


def test_activation_quant_rows_bit_exact():
    from aeo_quant_b200 import _capi as A
    lib = A.load()
    x = randn_bf16((67, 2816), 1.0, 3)
    x[5] = 0
    x[6, :7] = torch.tensor([1e-30, -3e4, 448.0, float("inf"), 0.0, -0.0, 2.0 ** -20])
    q = torch.empty(67, 2816, dtype=torch.uint8, device="cuda")
    sa = torch.empty(67, dtype=torch.float32, device="cuda")
    A.check(lib.aeoq_fp8_quantize_rows_gather(x.data_ptr(), 2816, None, None, 67, 2816, q.data_ptr(), 2816,
                                              sa.data_ptr(), A.stream_ptr(x.device)))
    qo, so = OQ.quantize_fp8_activation_rows(bf16_to_np(x))
    # inf / inf: NaN, whose sign bit differs between x86 (numpy) and the GPU;
    # NaN codes compare without the sign
    mine, ref = u8(q), qo
    nan = (ref & 0x7F) == 0x7F
    np.testing.assert_array_equal((mine & 0x7F) == 0x7F, nan)
    np.testing.assert_array_equal(mine[~nan], ref[~nan])
    np.testing.assert_array_equal(sa.cpu().numpy(), so.reshape(-1))


def test_activation_quant_gathers_rows():
    from aeo_quant_b200 import _capi as A
    lib = A.load()
    x = randn_bf16((10, 128), 1.0, 4)
    idx = torch.tensor([3, 3, 0, 9, 1], dtype=torch.int32, device="cuda")
    n = torch.tensor([4], dtype=torch.int32, device="cuda")
    q = torch.zeros(5, 128, dtype=torch.uint8, device="cuda")
    sa = torch.zeros(5, dtype=torch.float32, device="cuda")
    A.check(lib.aeoq_fp8_quantize_rows_gather(x.data_ptr(), 128, idx.data_ptr(), n.data_ptr(), 5, 128,
                                              q.data_ptr(), 128, sa.data_ptr(), A.stream_ptr(x.device)))
    qo, so = OQ.quantize_fp8_activation_rows(bf16_to_np(x)[[3, 3, 0, 9]])
    np.testing.assert_array_equal(u8(q)[:4], qo)
    np.testing.assert_array_equal(sa.cpu().numpy()[:4], so.reshape(-1))
    assert u8(q)[4].max() == 0   # rows past *n_rows untouched


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (37, 1408, 2816), (300, 2816, 704), (5, 256, 96)])
def test_fp8_linear_matches_oracle(M, N, K):
    from aeo_quant_b200.bridges.gemma4.moe_ops import fp8_linear
    from aeo_quant_b200.gpu import quant as Q
    x = randn_bf16((M, K), 1.0, 11)
    w = randn_bf16((N, K), 0.02, 12)
    wq, ws = Q.quantize_2d_to_fp8(w)
    sb = ws.reshape(1, N).float()
    y = fp8_linear(x, wq, sb)
    qx, sx = OQ.quantize_fp8_activation_rows(bf16_to_np(x))
    ref = fp8_scaled_mm(qx, sx, u8(wq.view(torch.uint8)), sb.cpu().numpy())
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    assert within_tol_or_ulp(bf16_to_np(y), ref)


@pytest.fixture(scope="module")
def golden_fp8(moe_golden):
    g = moe_golden
    E, twoI, H = g["f8/gate_up_proj"].shape
    t = lambda k: torch.from_numpy(g[k].copy()).cuda()
    return make_fp8_module(E, H, twoI // 2, t("f8/gate_up_proj").view(torch.float8_e4m3fn),
                           t("f8/gate_up_proj_scale"), t("f8/down_proj").view(torch.float8_e4m3fn),
                           t("f8/down_proj_scale"))


@pytest.mark.parametrize("T", [1, 7, 33])
def test_fp8_golden_forward(golden_fp8, moe_golden, T):
    g = moe_golden
    h = bits_to_bf16(g[f"f8/T{T}/hidden"])
    idx = torch.from_numpy(g[f"f8/T{T}/idx"]).cuda()
    w = bits_to_bf16(g[f"f8/T{T}/w"])
    y = golden_fp8(h, idx, w)
    ref = N.bf16_from_bits(g[f"f8/T{T}/out"])
    assert y.shape == h.shape and y.dtype == torch.bfloat16
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


@pytest.fixture(scope="module")
def full_fp8():
    """FP8 expert layer: 128 experts, H=2816, I=704, e4m3 rowwise."""
    from aeo_quant_b200.gpu import quant as Q
    E, H, I = 128, 2816, 704
    gq, gs = Q.quantize_3d_to_fp8(randn_bf16((E, 2 * I, H), 0.02, 300))
    dq, ds = Q.quantize_3d_to_fp8(randn_bf16((E, H, I), 0.02, 301))
    return make_fp8_module(E, H, I, gq, gs, dq, ds), (gq, gs, dq, ds)


# The composed forward re-quantizes the GeGLU rows to e4m3 (3 mantissa
# bits): a gate_up output one bf16 ulp away from the f64 oracle (f32
# accumulation order; about 1 in 10^4 outputs) can move one e4m3 code of its
# row by one step, which the down projection spreads over the output row.
# Each GEMM stage is held to TOL or one ulp on its own inputs
# (test_fp8_stages_full_size); the composed forward to MOE_TOL.
MOE_TOL = 1e-2


@pytest.mark.parametrize("T", [1, 16, 97])
def test_fp8_full_size_vs_oracle(full_fp8, T):
    m, (gq, gs, dq, ds) = full_fp8
    h = randn_bf16((T, 2816), 1.0, 40 + T)
    idx, w = routing(T, 128, 8, 50 + T)
    y = m(h, idx.cuda(), w.cuda())
    om = OM.FP8Experts(u8(gq.view(torch.uint8)), gs.float().cpu().numpy().reshape(128, 1, -1),
                       u8(dq.view(torch.uint8)), ds.float().cpu().numpy().reshape(128, 1, -1))
    ref = OM.fp8_experts_forward(om, bf16_to_np(h), idx.numpy(), bf16_to_np(w))
    assert max_rel_err(bf16_to_np(y), ref) <= MOE_TOL


def test_fp8_stages_full_size(full_fp8):
    """Each routed expert's gate_up GEMM, and its down GEMM on the GPU's own
    GeGLU rows, within TOL (or one bf16 ulp) of the oracle."""
    from aeo_quant_b200.bridges.gemma4.moe_ops import fp8_linear
    m, (gq, gs, dq, ds) = full_fp8
    T = 5
    h = randn_bf16((T, 2816), 1.0, 91)
    idx, _ = routing(T, 128, 8, 92)
    gqn, dqn = u8(gq.view(torch.uint8)), u8(dq.view(torch.uint8))
    gsn, dsn = gs.float().cpu().numpy().reshape(128, -1), ds.float().cpu().numpy().reshape(128, -1)
    for e in np.unique(idx.numpy()):
        rows = h[torch.from_numpy(np.nonzero((idx.numpy() == e).any(1))[0]).cuda()]
        gu = fp8_linear(rows, gq[e], gs[e].reshape(1, -1).float())
        gu_ref = OM.fp8_linear(bf16_to_np(rows), gqn[e], gsn[e])
        assert within_tol_or_ulp(bf16_to_np(gu), gu_ref)
        cur = OM.geglu(bf16_to_np(gu))
        d = fp8_linear(torch.from_numpy(cur).to(torch.bfloat16).cuda(), dq[e], ds[e].reshape(1, -1).float())
        assert within_tol_or_ulp(bf16_to_np(d), OM.fp8_linear(cur, dqn[e], dsn[e]))


def test_fp8_invalid_expert_is_skipped(golden_fp8):
    h = randn_bf16((3, 128), 1.0, 9)
    idx = torch.tensor([[0, 1, 2, 8], [8, 8, 3, 4], [5, 6, 7, 0]], device="cuda")
    w = torch.full((3, 4), 0.25, dtype=torch.bfloat16, device="cuda")
    y = golden_fp8(h, idx, w)
    y_ok = golden_fp8(h, torch.where(idx == 8, torch.zeros_like(idx), idx), torch.where(idx == 8, 0.0, w).to(torch.bfloat16))
    # id == num_experts contributes nothing (modeling.py:120-121); expert 0 with weight 0 adds zeros
    assert torch.equal(y, y_ok)


def test_fp8_scale_layouts_agree(full_fp8):
    """Checkpoint (E, N, 1) bf16 scales and the preconverted (E, 1, N) f32 ones give one result."""
    m, (gq, gs, dq, ds) = full_fp8
    h = randn_bf16((4, 2816), 1.0, 77)
    idx, w = routing(4, 128, 8, 78)
    y1 = m(h, idx.cuda(), w.cuda())
    m2 = make_fp8_module(128, 2816, 704, gq, gs, dq, ds)
    m2.gate_up_proj_scale = gs.clone()
    m2.down_proj_scale = ds.clone()
    assert torch.equal(y1, m2(h, idx.cuda(), w.cuda()))
