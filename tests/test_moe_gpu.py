"""Gemma4TextExpertsNVFP4 forwards on the GPU vs the oracle restatement of the
reference forwards, and vs the reference-generated golden outputs."""
import types

import numpy as np
import pytest
import torch

from helpers import TOL, bf16_to_np, bits_to_bf16, max_rel_err, randn_bf16, routing, u8
from oracle import moe as OM
from oracle import numerics as N

pytestmark = pytest.mark.gpu


def make_module(E, H, I, gp, gs, gt, dp, ds, dt):
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    cfg = types.SimpleNamespace(num_experts=E, hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")
    m = Gemma4TextExpertsNVFP4(cfg).cuda()
    m.gate_up_proj.copy_(gp)
    m.gate_up_proj_scale.copy_(gs)
    m.gate_up_proj_scale_2.copy_(gt)
    m.down_proj.copy_(dp)
    m.down_proj_scale.copy_(ds)
    m.down_proj_scale_2.copy_(dt)
    return m


@pytest.fixture(scope="module")
def golden_module(moe_golden):
    g = moe_golden
    t = lambda k, dt=torch.uint8: torch.from_numpy(g[k].copy()).view(dt).cuda()
    E, twoI, Hh = g["nv/gate_up_proj"].shape
    return make_module(E, Hh * 2, twoI // 2, t("nv/gate_up_proj"),
                       t("nv/gate_up_proj_scale").view(torch.float8_e4m3fn),
                       torch.tensor(g["nv/gate_up_proj_scale_2"][0]),
                       t("nv/down_proj"), t("nv/down_proj_scale").view(torch.float8_e4m3fn),
                       torch.tensor(g["nv/down_proj_scale_2"][0]))


@pytest.mark.parametrize("T", [1, 7, 33])
def test_golden_forward(golden_module, moe_golden, T):
    g = moe_golden
    h = bits_to_bf16(g[f"nv/T{T}/hidden"])
    idx = torch.from_numpy(g[f"nv/T{T}/idx"]).cuda()
    w = bits_to_bf16(g[f"nv/T{T}/w"])
    y = golden_module(h, idx, w)
    assert y.shape == h.shape and y.dtype == torch.bfloat16
    ref = N.bf16_from_bits(g[f"nv/T{T}/out"])
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


@pytest.fixture(scope="module")
def full_layer():
    """NVFP4 expert layer: 128 experts, H=2816, I=704, NVFP4 per projection."""
    from aeo_quant_b200.gpu import quant as Q
    E, H, I = 128, 2816, 704
    wgu = randn_bf16((E, 2 * I, H), 0.02, 100)
    gp, gs, gt = Q.quantize_3d_to_nvfp4(wgu)
    del wgu
    wd = randn_bf16((E, H, I), 0.02, 101)
    dp, ds, dt = Q.quantize_3d_to_nvfp4(wd)
    del wd
    m = make_module(E, H, I, gp, gs, gt.float(), dp, ds, dt.float())
    return m


def oracle_module(m, experts):
    """Oracle view holding only the experts that the routing touches."""
    sel = sorted(set(int(e) for e in experts))
    remap = {e: i for i, e in enumerate(sel)}
    ix = torch.tensor(sel, device="cuda")
    om = OM.NVFP4Experts(u8(m.gate_up_proj[ix]), u8(m.gate_up_proj_scale[ix]), float(m.gate_up_proj_scale_2),
                         u8(m.down_proj[ix]), u8(m.down_proj_scale[ix]), float(m.down_proj_scale_2))
    return om, remap


@pytest.mark.parametrize("B,seed", [(1, 0), (1, 1), (1, 2), (4, 3), (16, 4), (64, 5), (200, 6)])
def test_full_size_vs_oracle(full_layer, B, seed):
    m = full_layer
    h = randn_bf16((B, 2816), 1.0, 200 + seed)
    idx, w = routing(B, 128, 8, 300 + seed)
    y = m(h, idx.cuda(), w.cuda())
    om, remap = oracle_module(m, idx.flatten().tolist())
    idx_r = np.vectorize(remap.get)(idx.numpy())
    ref = OM.nvfp4_experts_forward(om, bf16_to_np(h), idx_r, bf16_to_np(w))
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_decode_int32_ids_and_repeatable(full_layer):
    m = full_layer
    h = randn_bf16((1, 2816), 1.0, 400)
    idx, w = routing(1, 128, 8, 401)
    y64 = m(h, idx.cuda(), w.cuda())
    y32 = m(h, idx.to(torch.int32).cuda(), w.cuda())
    y64b = m(h, idx.cuda(), w.cuda())
    assert torch.equal(y64, y32) and torch.equal(y64, y64b)


def test_decode_graph_capture(full_layer):
    m = full_layer
    h = randn_bf16((1, 2816), 1.0, 500)
    idx, w = routing(1, 128, 8, 501)
    idx, w = idx.cuda(), w.cuda()
    ref = m(h, idx, w)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        m(h, idx, w)
        with torch.cuda.graph(g, stream=s):
            out = m(h, idx, w)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_decode_three_launch_path_matches_fused(full_layer):
    """The chained three-launch decode (used when a shape does not fit the
    cooperative kernel's shared-memory plan) gives the same bits."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    for seed in range(3):
        h = randn_bf16((1, 2816), 1.0, 600 + seed)
        idx, w = routing(1, 128, 8, 700 + seed)
        args = (h, idx.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
                m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
        assert torch.equal(moe_ops.nvfp4_decode(*args, fused=True), moe_ops.nvfp4_decode(*args, fused=False))


@pytest.mark.parametrize("path", ["stream", "tc", "fused", "chained"])
def test_decode_invalid_expert_contributes_zero(full_layer, path):
    """An id outside [0, E) adds nothing (the reference skips id == E). Its
    GeGLU row is zero, so the shared tensor scale of the other seven is
    unchanged: the output is the oracle's forward over the seven valid slots."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    h = randn_bf16((1, 2816), 1.0, 800)
    idx, w = routing(1, 128, 8, 801)
    idx2 = idx.clone()
    idx2[0, 3] = 128
    args = (h, idx2.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
            m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
    y = moe_ops.nvfp4_decode(*args, path=path)
    om, remap = oracle_module(m, [e for e in idx[0].tolist() if e != idx[0, 3].item()])
    keep = [j for j in range(8) if j != 3]
    ids_r = np.array([[remap[int(idx[0, j])] for j in keep]])
    ref = OM.nvfp4_experts_forward(om, bf16_to_np(h), ids_r, bf16_to_np(w)[:, keep])
    assert max_rel_err(bf16_to_np(y), ref) <= TOL


@pytest.mark.parametrize("path", ["stream", "tc", "fused", "chained"])
def test_decode_each_path_vs_oracle(full_layer, path):
    """Every one-token kernel against the oracle on the same inputs."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    for seed in range(3):
        h = randn_bf16((1, 2816), 1.0, 1500 + seed)
        idx, w = routing(1, 128, 8, 1600 + seed)
        args = (h, idx.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
                m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
        y = moe_ops.nvfp4_decode(*args, path=path)
        om, remap = oracle_module(m, idx.flatten().tolist())
        idx_r = np.vectorize(remap.get)(idx.numpy())
        ref = OM.nvfp4_experts_forward(om, bf16_to_np(h), idx_r, bf16_to_np(w))
        assert max_rel_err(bf16_to_np(y), ref) <= TOL, (path, seed)


def test_decode_stream_repeated_calls_reuse_workspace(full_layer):
    """The streamed kernel's counters reset themselves: many calls in a row
    on one workspace give the same bits as a fresh run."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    h = randn_bf16((1, 2816), 1.0, 1700)
    idx, w = routing(1, 128, 8, 1701)
    args = (h, idx.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
            m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
    ref = moe_ops.nvfp4_decode(*args, path="stream")
    outs = [moe_ops.nvfp4_decode(*args, path="stream") for _ in range(50)]
    assert all(torch.equal(o, ref) for o in outs)


def test_grouped_one_token_semantics_matches_fused(full_layer):
    """The device-grouped pipeline run with one-token semantics (shared down
    scale, f32 combine) agrees with the cooperative decode kernel."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    for seed in range(3):
        h = randn_bf16((1, 2816), 1.0, 1100 + seed)
        idx, w = routing(1, 128, 8, 1200 + seed)
        args = (h, idx.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
                m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
        y1 = moe_ops.nvfp4_decode(*args)
        y2 = moe_ops.nvfp4_experts_grouped(*args, one_token_semantics=True)
        assert max_rel_err(bf16_to_np(y2), bf16_to_np(y1)) <= TOL


def test_decode_tensor_core_path_matches_cuda_core(full_layer):
    """Tensor-core one-token decode vs the cooperative CUDA-core kernel: both
    round once from f32 sums of exact block products."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    m = full_layer
    for seed in range(4):
        h = randn_bf16((1, 2816), 1.0, 1300 + seed)
        idx, w = routing(1, 128, 8, 1400 + seed)
        args = (h, idx.cuda(), w.cuda(), m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
                m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
        y_tc = moe_ops.nvfp4_decode(*args, path="tc")
        y_cc = moe_ops.nvfp4_decode(*args, path="fused")
        assert max_rel_err(bf16_to_np(y_tc), bf16_to_np(y_cc)) <= TOL
