"""The torch restatement (oracle/torch_port.py) against the numpy oracle
and the reference-generated golden outputs, on the CPU: quantizer bytes bit
for bit, expert forwards within the output tolerance. This pins the port
that bench.py times as the CPU baseline and that the stack test runs on the
GPU as its checker."""
import numpy as np
import pytest
import torch

from helpers import TOL, max_rel_err
from oracle import moe as OM
from oracle import numerics as N
from oracle import quant as OQ
from oracle import torch_port as TP


def _bf16(a):
    return torch.from_numpy(N.bf16_bits(np.asarray(a, np.float32)).view(np.int16).copy()).view(torch.bfloat16)


@pytest.mark.parametrize("shape,std,seed", [((37, 256), 1.0, 0), ((8, 704), 0.3, 1), ((4, 2816), 1e-3, 2)])
def test_quantizer_bit_exact(shape, std, seed):
    rng = np.random.default_rng(seed)
    x = N.bf16(rng.standard_normal(shape).astype(np.float32) * std)
    x[0, :16] = 0.0                                   # a zero block
    x[1, 16:32] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, 0, -0.0, 1e-30, 3, 4, 6]
    p, s, ts = OQ.quantize_nvfp4(x)
    tp, tsf, tts = TP.quantize_nvfp4(_bf16(x))
    assert np.array_equal(tp.numpy(), p) and np.array_equal(tsf.numpy(), s)
    assert float(tts) == float(np.ravel(ts)[0])


def test_gemm_matches_oracle():
    rng = np.random.default_rng(3)
    a = N.bf16(rng.standard_normal((33, 512)).astype(np.float32))
    w = N.bf16(rng.standard_normal((128, 512)).astype(np.float32) * 0.02)
    ap, asf, ats = OQ.quantize_nvfp4(a)
    wp, wsf, wts = OQ.quantize_nvfp4(w)
    ref = OM.nvfp4_gemm(ap, asf, ats, wp, wsf, wts)
    t = lambda v: torch.from_numpy(np.ascontiguousarray(v))
    y = TP.nvfp4_gemm(t(ap), t(asf), float(np.ravel(ats)[0]), t(wp), t(wsf), float(np.ravel(wts)[0])).to(torch.float32).numpy()
    assert max_rel_err(y, ref) <= TOL
    y64 = TP.nvfp4_gemm(t(ap), t(asf), float(np.ravel(ats)[0]), t(wp), t(wsf), float(np.ravel(wts)[0]), exact=True).to(torch.float32).numpy()
    assert np.array_equal(N.bf16_bits(y64), N.bf16_bits(ref))


@pytest.mark.parametrize("T", [1, 7, 33])
def test_forward_matches_golden(moe_golden, T):
    g = moe_golden
    m = TP.Experts(torch.from_numpy(g["nv/gate_up_proj"]), torch.from_numpy(g["nv/gate_up_proj_scale"]),
                   float(g["nv/gate_up_proj_scale_2"][0]), torch.from_numpy(g["nv/down_proj"]),
                   torch.from_numpy(g["nv/down_proj_scale"]), float(g["nv/down_proj_scale_2"][0]))
    h = torch.from_numpy(g[f"nv/T{T}/hidden"].view(np.int16).copy()).view(torch.bfloat16)
    w = torch.from_numpy(g[f"nv/T{T}/w"].view(np.int16).copy()).view(torch.bfloat16)
    idx = torch.from_numpy(g[f"nv/T{T}/idx"])
    ref = N.bf16_from_bits(g[f"nv/T{T}/out"])
    y = TP.forward(m, h, idx, w).to(torch.float32).numpy()
    assert max_rel_err(y, ref) <= TOL
    # with float64 sums the port reproduces the golden outputs bit for bit
    y64 = TP.forward(m, h, idx, w, exact=True).to(torch.float32).numpy()
    assert np.array_equal(N.bf16_bits(y64), g[f"nv/T{T}/out"])
