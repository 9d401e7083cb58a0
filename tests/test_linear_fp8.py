"""LinearFP8: the module's parameter/buffer layout on the CPU (the names,
shapes and dtypes a checkpoint holds), and on the GPU ``from_linear`` plus
forward against the oracle's ``_fp8_linear`` restatement, including widths
that are not a multiple of 128, a bias, and leading batch dimensions."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from helpers import bf16_to_np, randn_bf16, u8, within_tol_or_ulp
from oracle import moe as OM
from oracle import numerics as NU
from oracle import quant as OQ


def test_layout_cpu():
    from aeo_quant_b200.bridges.gemma4.linear_fp8 import LinearFP8
    m = LinearFP8(2816, 2112, bias=True)
    sd = m.state_dict()
    assert set(sd) == {"weight", "weight_scale", "bias"}
    assert sd["weight"].shape == (2112, 2816) and sd["weight"].dtype == torch.float8_e4m3fn
    assert sd["weight_scale"].shape == (1, 2112) and sd["weight_scale"].dtype == torch.float32
    assert sd["bias"].dtype == torch.bfloat16 and not m.weight.requires_grad
    assert "dtype=float8_e4m3fn" in repr(m)
    assert set(LinearFP8(64, 128).state_dict()) == {"weight", "weight_scale"}


@pytest.mark.gpu
@pytest.mark.parametrize("shape,N,K,bias", [((7,), 2112, 2816, False), ((2, 5), 256, 128, True),
                                            ((33,), 2816, 2112, True), ((1,), 96, 64, False)])
def test_from_linear_forward_vs_oracle(shape, N, K, bias):
    from aeo_quant_b200.bridges.gemma4.linear_fp8 import LinearFP8
    lin = nn.Linear(K, N, bias=bias).to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(randn_bf16((N, K), 0.02, 21))
        if bias:
            lin.bias.copy_(randn_bf16((N,), 0.1, 22))
    m = LinearFP8.from_linear(lin)
    wq, ws = OQ.quantize_fp8_rows(bf16_to_np(lin.weight.detach()))
    np.testing.assert_array_equal(u8(m.weight.detach().view(torch.uint8)), wq)
    np.testing.assert_array_equal(m.weight_scale.cpu().numpy().reshape(-1), ws.reshape(-1))
    x = randn_bf16((*shape, K), 1.0, 23)
    with torch.no_grad():
        y = m(x)
        y2 = m(x)                                   # second call: cached padded copy
    assert y.shape == (*shape, N) and y.dtype == torch.bfloat16 and y.is_contiguous()
    assert torch.equal(y, y2)
    ref = OM.fp8_linear(bf16_to_np(x).reshape(-1, K), wq, ws.reshape(1, N))
    if bias:
        ref = NU.bf16(ref + bf16_to_np(lin.bias.detach())[None, :])
    assert within_tol_or_ulp(bf16_to_np(y).reshape(-1, N), ref)
