"""Pin the numpy oracle against fixtures produced by the reference itself."""
import json
import hashlib
import os

import numpy as np
import pytest

from oracle import moe as OM
from oracle import numerics as N
from oracle import quant as OQ

from conftest import GOLDEN


def bf(bits):
    return N.bf16_from_bits(np.asarray(bits, np.uint16))


def test_fp4_rounding_table(quant_golden):
    x = quant_golden["fp4_round_in"]
    np.testing.assert_array_equal(N.fp4_nibble(x), quant_golden["fp4_round_out"])


@pytest.mark.parametrize("i", range(11))
def test_nvfp4_2d_cases(quant_golden, i):
    names = list(quant_golden["nvfp4_names"])
    if i >= len(names):
        pytest.skip("fewer cases")
    n = names[i]
    x = bf(quant_golden[f"nvfp4/{n}/x"])
    p, s, t = OQ.quantize_nvfp4(x, "bf16")
    np.testing.assert_array_equal(p, quant_golden[f"nvfp4/{n}/packed"])
    np.testing.assert_array_equal(s, quant_golden[f"nvfp4/{n}/sf"])
    assert N.bf16_bits(t)[()] == quant_golden[f"nvfp4/{n}/ts"][0]
    deq = OQ.dequant_nvfp4(p, s, t)
    np.testing.assert_array_equal(N.bf16_bits(deq), quant_golden[f"nvfp4/{n}/dequant"])


def test_nvfp4_f32_input(quant_golden):
    x = quant_golden["nvfp4_f32/x"]
    p, s, t = OQ.quantize_nvfp4(x, "f32")
    np.testing.assert_array_equal(p, quant_golden["nvfp4_f32/packed"])
    np.testing.assert_array_equal(s, quant_golden["nvfp4_f32/sf"])
    assert np.float32(t) == quant_golden["nvfp4_f32/ts"][0]


def test_nvfp4_3d(quant_golden):
    x = bf(quant_golden["nvfp4_3d/x"])
    p, s, t = OQ.quantize_nvfp4(x, "bf16")
    np.testing.assert_array_equal(p, quant_golden["nvfp4_3d/packed"])
    np.testing.assert_array_equal(s, quant_golden["nvfp4_3d/sf"])
    assert N.bf16_bits(t)[()] == quant_golden["nvfp4_3d/ts"][0]


def test_fp8_every_bf16_value(quant_golden):
    x = bf(np.arange(65536, dtype=np.uint32).astype(np.uint16)).reshape(-1, 1)
    q, s = OQ.quantize_fp8_rows(x)
    gq = quant_golden["fp8_all/codes"]
    gs = quant_golden["fp8_all/scale"]
    sb = N.bf16_bits(s.reshape(-1))
    # NaN payloads may differ in bits; compare NaN-ness there.
    nan_s = np.isnan(bf(gs))
    np.testing.assert_array_equal(np.isnan(s.reshape(-1)), nan_s)
    np.testing.assert_array_equal(sb[~nan_s], gs[~nan_s])
    np.testing.assert_array_equal(q.reshape(-1), gq)


def test_fp8_3d(quant_golden):
    x = bf(quant_golden["fp8_3d/x"])
    q, s = OQ.quantize_fp8_rows(x)
    np.testing.assert_array_equal(q, quant_golden["fp8_3d/codes"])
    np.testing.assert_array_equal(N.bf16_bits(s), quant_golden["fp8_3d/scale"])


def test_fp8_activation_rows(quant_golden):
    x = bf(quant_golden["fp8_act/x"])
    q, sa = OQ.quantize_fp8_activation_rows(x)
    np.testing.assert_array_equal(q, quant_golden["fp8_act/codes"])
    np.testing.assert_array_equal(sa.reshape(-1), quant_golden["fp8_act/scale"])


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    v = N.e4m3_decode(codes)
    back = N.e4m3_encode(v)
    ok = ~np.isnan(v)
    # +-0 both map to themselves
    np.testing.assert_array_equal(back[ok], codes[ok])


def test_e4m3_matches_torch_dense_sweep():
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.randn(200000, generator=g) * s for s in (1e-3, 0.1, 1.0, 30.0, 300.0)])
    x = torch.cat([x, torch.tensor([464.0, 463.9, 464.1, 479.9, 480.0, 448.0, -464.0, 2.0 ** -10,
                                    3 * 2.0 ** -11, float("inf"), float("-inf"), float("nan")])])
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    mine = N.e4m3_encode(x.numpy())
    np.testing.assert_array_equal(mine & 0x7F == 0x7F, ref & 0x7F == 0x7F)
    ok = (ref & 0x7F) != 0x7F
    np.testing.assert_array_equal(mine[ok], ref[ok])


def test_config0_hashes():
    torch = pytest.importorskip("torch")
    with open(os.path.join(GOLDEN, "config0_hashes.json")) as f:
        h = json.load(f)
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(1408, 2816, generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(128, 2816, generator=g).to(torch.bfloat16)
    for name, t in (("W", W), ("X", X)):
        bits = t.view(torch.int16).numpy().view(np.uint16)
        assert hashlib.sha256(bits.tobytes()).hexdigest() == h[name]["input"]
        p, s, ts = OQ.quantize_nvfp4(bf(bits), "bf16")
        assert hashlib.sha256(p.tobytes()).hexdigest() == h[name]["packed"]
        assert hashlib.sha256(s.tobytes()).hexdigest() == h[name]["sf"]
        assert int(N.bf16_bits(ts).reshape(-1)[0]) == h[name]["ts_bits"]


def _nv_module(g):
    return OM.NVFP4Experts(g["nv/gate_up_proj"], g["nv/gate_up_proj_scale"],
                           g["nv/gate_up_proj_scale_2"][0], g["nv/down_proj"],
                           g["nv/down_proj_scale"], g["nv/down_proj_scale_2"][0])


@pytest.mark.parametrize("T", [1, 7, 33])
def test_nvfp4_experts_forward(moe_golden, T):
    g = moe_golden
    m = _nv_module(g)
    y = OM.nvfp4_experts_forward(m, bf(g[f"nv/T{T}/hidden"]), g[f"nv/T{T}/idx"],
                                 bf(g[f"nv/T{T}/w"]))
    ref = bf(g[f"nv/T{T}/out"])
    np.testing.assert_array_equal(N.bf16_bits(y), N.bf16_bits(ref))


@pytest.mark.parametrize("T", [1, 7, 33])
def test_fp8_experts_forward(moe_golden, T):
    g = moe_golden
    m = OM.FP8Experts(g["f8/gate_up_proj"], g["f8/gate_up_proj_scale"], g["f8/down_proj"],
                      g["f8/down_proj_scale"])
    y = OM.fp8_experts_forward(m, bf(g[f"f8/T{T}/hidden"]), g[f"f8/T{T}/idx"],
                               bf(g[f"f8/T{T}/w"]))
    ref = bf(g[f"f8/T{T}/out"])
    np.testing.assert_array_equal(N.bf16_bits(y), N.bf16_bits(ref))
