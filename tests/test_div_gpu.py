"""The library's correctly rounded division against the compiler's
__fdiv_rn, bit for bit, over the quantizers' whole operand domains."""
import pytest
import torch

from aeo_quant_b200 import _capi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("domain", [0, 1, 2])
def test_div_rn_matches_fdiv_rn(domain):
    lib = _capi.load()
    mism = torch.zeros(1, dtype=torch.int64, device="cuda")
    ex = torch.zeros(17, dtype=torch.float32, device="cuda")
    rc = lib.aeoq_selftest_div_rn(domain, mism.data_ptr(), ex.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.aeoq_last_error()
    torch.cuda.synchronize()
    a, b, got, want = ex[:4].tolist()
    assert mism.item() == 0, f"{mism.item()} mismatches, first: {a!r} / {b!r} -> {got!r}, want {want!r}"


def test_block_quantizer_matches_division_formula():
    lib = _capi.load()
    mism = torch.zeros(1, dtype=torch.int64, device="cuda")
    ex = torch.zeros(17, dtype=torch.float32, device="cuda")
    rc = lib.aeoq_selftest_div_rn(3, mism.data_ptr(), ex.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.aeoq_last_error()
    torch.cuda.synchronize()
    assert mism.item() == 0, f"{mism.item()} blocks differ; first: ts={ex[0].item()!r} x={ex[1:].tolist()}"
