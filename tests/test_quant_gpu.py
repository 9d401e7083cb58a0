"""Quantizers on the GPU vs the reference-pinned oracle and golden fixtures:
bit-exact packed bytes, e4m3 scales and tensor scales."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import bits_to_bf16, u8
from oracle import numerics as N
from oracle import quant as OQ

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Q():
    from aeo_quant_b200.gpu import quant
    return quant


def _ts_bits(t):
    return int(t.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)[0])


def test_golden_2d_cases(Q, quant_golden):
    for n in list(quant_golden["nvfp4_names"]):
        x = bits_to_bf16(quant_golden[f"nvfp4/{n}/x"])
        p, s, t = Q.quantize_2d_to_nvfp4(x)
        assert p.dtype == torch.uint8 and s.dtype == torch.float8_e4m3fn and t.dtype == torch.bfloat16
        assert t.ndim == 0
        np.testing.assert_array_equal(u8(p), quant_golden[f"nvfp4/{n}/packed"], err_msg=n)
        np.testing.assert_array_equal(u8(s), quant_golden[f"nvfp4/{n}/sf"], err_msg=n)
        assert _ts_bits(t) == quant_golden[f"nvfp4/{n}/ts"][0], n
        d = Q.dequant_2d_from_nvfp4(p, s, t)
        np.testing.assert_array_equal(d.view(torch.int16).cpu().numpy().view(np.uint16),
                                      quant_golden[f"nvfp4/{n}/dequant"], err_msg=n)


def test_golden_f32_and_3d(Q, quant_golden):
    x = torch.from_numpy(quant_golden["nvfp4_f32/x"]).cuda()
    p, s, t = Q.quantize_2d_to_nvfp4(x)
    assert t.dtype == torch.float32
    np.testing.assert_array_equal(u8(p), quant_golden["nvfp4_f32/packed"])
    np.testing.assert_array_equal(u8(s), quant_golden["nvfp4_f32/sf"])
    assert float(t) == float(quant_golden["nvfp4_f32/ts"][0])
    x3 = bits_to_bf16(quant_golden["nvfp4_3d/x"])
    p, s, t = Q.quantize_3d_to_nvfp4(x3)
    assert p.shape == (3, 64, 64) and s.shape == (3, 64, 8)
    np.testing.assert_array_equal(u8(p), quant_golden["nvfp4_3d/packed"])
    np.testing.assert_array_equal(u8(s), quant_golden["nvfp4_3d/sf"])
    assert _ts_bits(t) == quant_golden["nvfp4_3d/ts"][0]


def test_config0_hashes_multi_cta_path(Q):
    """W[1408,2816] takes the two-launch (grid amax) path."""
    with open(os.path.join(GOLDEN, "config0_hashes.json")) as f:
        h = json.load(f)
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(1408, 2816, generator=g) * 0.02).to(torch.bfloat16).cuda()
    X = torch.randn(128, 2816, generator=g).to(torch.bfloat16).cuda()
    for name, t in (("W", W), ("X", X)):
        p, s, ts = Q.quantize_2d_to_nvfp4(t)
        assert hashlib.sha256(u8(p).tobytes()).hexdigest() == h[name]["packed"], name
        assert hashlib.sha256(u8(s).tobytes()).hexdigest() == h[name]["sf"], name
        assert _ts_bits(ts) == h[name]["ts_bits"], name


@pytest.mark.parametrize("shape,std,seed", [((16, 1408, 2816), 0.02, 3), ((7, 1408, 704), 1.0, 4),
                                            ((1, 16), 1.0, 5), ((3, 5, 48), 3.0, 6)])
def test_random_vs_oracle(Q, shape, std, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)
    if len(shape) == 2:
        p, s, t = Q.quantize_2d_to_nvfp4(x.cuda())
    else:
        p, s, t = Q.quantize_3d_to_nvfp4(x.cuda())
    # oracle on a bounded sample of rows (same global tensor scale)
    xf = x.float().numpy().reshape(-1, shape[-1])
    ts = OQ.nvfp4_tensor_scale(np.max(np.abs(xf)))
    assert _ts_bits(t) == int(N.bf16_bits(ts).reshape(-1)[0])
    rows = np.unique(np.linspace(0, xf.shape[0] - 1, num=min(512, xf.shape[0])).astype(int))
    op, osf, _ = OQ.quantize_nvfp4(xf[rows], ts=ts)
    np.testing.assert_array_equal(u8(p).reshape(xf.shape[0], -1)[rows], op)
    np.testing.assert_array_equal(u8(s).reshape(xf.shape[0], -1)[rows], osf)


def test_strided_input(Q):
    x = torch.randn(64, 256, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).cuda()
    view = x[:, :128]                       # row stride 256, not contiguous
    p, s, t = Q.quantize_2d_to_nvfp4(view)
    p2, s2, t2 = Q.quantize_2d_to_nvfp4(view.contiguous())
    assert torch.equal(p, p2) and torch.equal(s.view(torch.uint8), s2.view(torch.uint8))


def test_fp8_every_bf16_value(Q, quant_golden):
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).reshape(-1, 1).cuda()
    q, s = Q.quantize_2d_to_fp8(allbf)
    assert q.dtype == torch.float8_e4m3fn and s.dtype == torch.bfloat16 and s.shape == (65536, 1)
    np.testing.assert_array_equal(u8(q).reshape(-1), quant_golden["fp8_all/codes"])
    gs = quant_golden["fp8_all/scale"]
    sb = s.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    nan = np.isnan(N.bf16_from_bits(gs))
    np.testing.assert_array_equal(np.isnan(N.bf16_from_bits(sb)), nan)
    np.testing.assert_array_equal(sb[~nan], gs[~nan])


def test_fp8_3d_and_activation(Q, quant_golden):
    x3 = bits_to_bf16(quant_golden["fp8_3d/x"])
    q, s = Q.quantize_3d_to_fp8(x3)
    np.testing.assert_array_equal(u8(q), quant_golden["fp8_3d/codes"])
    np.testing.assert_array_equal(s.view(torch.int16).cpu().numpy().view(np.uint16), quant_golden["fp8_3d/scale"])
    xa = bits_to_bf16(quant_golden["fp8_act/x"])
    q, sa = Q.quantize_fp8_activation_rows(xa)
    np.testing.assert_array_equal(u8(q), quant_golden["fp8_act/codes"])
    np.testing.assert_array_equal(sa.cpu().numpy().reshape(-1), quant_golden["fp8_act/scale"])


def test_graph_capturable(Q):
    x = torch.randn(8, 704, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).cuda()
    p0, s0, t0 = Q.quantize_2d_to_nvfp4(x)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        Q.quantize_2d_to_nvfp4(x)   # warm-up on the capture stream
        with torch.cuda.graph(g, stream=s):
            p, sf, t = Q.quantize_2d_to_nvfp4(x)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(p, p0) and torch.equal(t, t0)
