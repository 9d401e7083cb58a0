"""The fused Gemma-4 router kernel against the router oracle and against
HF transformers' eager Gemma4TextRouter on the same GPU."""
import numpy as np
import pytest
import torch

from helpers import bf16_to_np, check_router
from oracle import router as OR
from test_router_oracle import hf_router, oracle_of

pytestmark = pytest.mark.gpu


def fused(r):
    """A copy of HF router ``r`` with the fused forward installed."""
    import copy
    from aeo_quant_b200.bridges.gemma4.loader import swap_routers
    f = copy.deepcopy(r)
    assert swap_routers(torch.nn.Sequential(f)) == 1
    return f


@pytest.mark.parametrize("H,E,k,T", [(2816, 128, 8, 1), (2816, 128, 8, 7), (2816, 128, 8, 8), (2816, 128, 8, 9),
                                     (2816, 128, 8, 64), (2816, 128, 8, 300), (512, 16, 4, 5), (1024, 256, 32, 17),
                                     (6144, 64, 8, 3), (2816, 128, 8, 33)])
def test_router_vs_oracle(H, E, k, T, monkeypatch):
    from aeo_quant_b200.bridges.gemma4 import router as R
    monkeypatch.setattr(R, "FUSED_MAX_TOKENS", 1 << 30)   # the kernel at every token count
    r = hf_router(H, E, k, 11, 0.5).cuda()
    f = fused(r)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(T)) * 2.0).to(torch.bfloat16).cuda()
    with torch.no_grad():
        p, w, i = f(x)
    assert p.shape == (T, E) and w.shape == (T, k) and i.shape == (T, k) and i.dtype == torch.int64
    op, ow, oi = oracle_of(r, x)
    differ = check_router(bf16_to_np(p), bf16_to_np(w), i.cpu().numpy(), op, ow, oi)
    assert differ <= max(1, T // 8)


@pytest.mark.parametrize("std", [0.02, 0.5])
def test_router_vs_hf_eager_on_gpu(std):
    r = hf_router(2816, 128, 8, 12, std).cuda()
    f = fused(r)
    x = (torch.randn(32, 2816, generator=torch.Generator().manual_seed(5))).to(torch.bfloat16).cuda()
    with torch.no_grad():
        p, w, i = f(x)
        hp, hw, hi = r(x)
    differ = check_router(bf16_to_np(p), bf16_to_np(w), i.cpu().numpy(), bf16_to_np(hp), bf16_to_np(hw),
                          hi.cpu().numpy())
    if std >= 0.5:
        assert differ <= 4


def test_router_strided_input_and_repeatable():
    r = hf_router(2816, 128, 8, 13, 0.5).cuda()
    f = fused(r)
    big = torch.randn(6, 2 * 2816, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).cuda()
    x = big[:, :2816]                      # row stride 2 * H
    with torch.no_grad():
        a = f(x)
        b = f(x.contiguous())
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_router_rejects_unsupported_shapes():
    r = hf_router(2816, 12, 4, 14, 0.5).cuda()     # 12 experts: not a multiple of 8
    f = fused(r)
    x = torch.randn(2, 2816, device="cuda").to(torch.bfloat16)
    with pytest.raises(ValueError, match="multiple of 8"):
        f(x)
    with pytest.raises(ValueError, match="bfloat16"):
        f(x.float())


def test_router_large_batches_take_hf_forward():
    """Above FUSED_MAX_TOKENS the swapped router runs HF's eager forward
    (faster there): identical outputs to the unswapped module."""
    from aeo_quant_b200.bridges.gemma4 import router as R
    r = hf_router(2816, 128, 8, 15, 0.5).cuda()
    f = fused(r)
    x = torch.randn(R.FUSED_MAX_TOKENS + 1, 2816, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        for u, v in zip(f(x), r(x)):
            assert torch.equal(u, v)
