"""Generate the golden fixtures from the aeo_quant reference itself.

Run in a container that has the reference source tree (it is imported, never
copied)::

    python tests/golden/make_golden.py /path/to/aeo-quant

Every fixture is produced by the reference's own code:

* ``quant_golden.npz`` — ``quantize_2d_to_nvfp4`` / ``quantize_3d_to_nvfp4`` /
  ``quantize_2d_to_fp8`` / ``quantize_3d_to_fp8`` / ``dequant_2d_from_nvfp4``
  (``src/aeo_quant/gpu/quant.py``) and ``_round_to_fp4_e2m1`` on seeded and
  hand-built inputs, plus the per-row FP8 activation quant of
  ``Gemma4TextExpertsFP8._fp8_linear`` captured at its ``torch._scaled_mm``
  call (``bridges/gemma4/modeling.py:101-108``).
* ``moe_golden.npz`` — the reference ``Gemma4TextExpertsNVFP4.forward``
  (decode and prefill branches) and ``Gemma4TextExpertsFP8.forward`` run on
  CPU. Their GEMMs are third-party kernels (Triton ``tl.dot_scaled``,
  cuBLASLt ``_scaled_mm``) that cannot run here; they are replaced at the call
  site by the published contract (exact block-scaled operands, float64 dot,
  one float32 rounding, ``alpha`` epilogue, bf16 output), so these fixtures
  pin the reference's routing, casts, re-quantization and combine.
* ``config0_hashes.json`` — SHA-256 of the reference quantizer outputs for
  the single-linear case (W[1408,2816] ~ N(0,0.02) and X[128,2816] ~ N(0,1),
  seed 0), too large to store in full.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def u8(t):
    return t.contiguous().view(torch.uint8).numpy().copy()


def bf16bits(t):
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def gen_bf16(shape, std, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def tie_row():
    # amax 10.5 -> ts = 10.5/2688 = 2^-8 exactly; block max 2688 -> scale 448,
    # so x*256/448 lands exactly on every FP4 midpoint and grid value.
    q = [6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -0.75, -1.25, -1.75,
         -2.5, -3.5, -5.0, 0.0]
    return torch.tensor([v * 1.75 for v in q] * 2, dtype=torch.bfloat16).reshape(1, 32)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from aeo_quant.gpu import quant as Q

    out = {}
    # --- FP4 rounding table ---------------------------------------------
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75,
                         0.0, -0.0, 0.2, 0.3, 0.7, 0.8, 1.2, 1.3, 1.7, 1.8, 2.4, 2.6,
                         3.4, 3.6, 4.9, 5.1, -5.9, float("nan"), -1e-30],
                        dtype=torch.float32)
    out["fp4_round_in"] = ties.numpy()
    out["fp4_round_out"] = Q._round_to_fp4_e2m1(ties).numpy()

    # --- NVFP4 2D cases ---------------------------------------------------
    cases = {
        "rand_1x16": gen_bf16((1, 16), 1.0, 1),
        "rand_3x32": gen_bf16((3, 32), 0.02, 2),
        "rand_8x704": gen_bf16((8, 704), 1.0, 3),
        "rand_1x2816": gen_bf16((1, 2816), 1.0, 4),
        "rand_64x2816": gen_bf16((64, 2816), 0.02, 5),
        "zeros_2x32": torch.zeros(2, 32, dtype=torch.bfloat16),
        "ties_1x32": tie_row(),
    }
    tiny = gen_bf16((4, 64), 1.0, 6)
    tiny[1, :16] = tiny[1, :16] * 1e-6      # a block whose scale underflows to 0
    tiny[2, 16:32] = 0.0                     # an all-zero block in a non-zero tensor
    tiny[3, 5] = -tiny[3, 5].abs() * 1e-4    # a small negative that rounds to -0
    cases["tinyblocks_4x64"] = tiny
    big = gen_bf16((2, 48), 1.0, 7)
    big[0, 3] = 3.0e38                       # near the bf16 maximum
    cases["huge_2x48"] = big
    wide = gen_bf16((5, 48), 1.0, 8)
    wide[:, ::7] *= 300.0                    # wide dynamic range inside blocks
    cases["wide_5x48"] = wide
    names = sorted(cases)
    out["nvfp4_names"] = np.array(names)
    for n in names:
        x = cases[n]
        p, s, t = Q.quantize_2d_to_nvfp4(x)
        out[f"nvfp4/{n}/x"] = bf16bits(x)
        out[f"nvfp4/{n}/packed"] = p.numpy()
        out[f"nvfp4/{n}/sf"] = u8(s)
        out[f"nvfp4/{n}/ts"] = bf16bits(t.reshape(1))
        out[f"nvfp4/{n}/dequant"] = bf16bits(Q.dequant_2d_from_nvfp4(p, s, t))
    # float32 input keeps a float32 tensor scale
    xf = torch.randn(4, 32, generator=torch.Generator().manual_seed(9))
    p, s, t = Q.quantize_2d_to_nvfp4(xf)
    out["nvfp4_f32/x"] = xf.numpy()
    out["nvfp4_f32/packed"] = p.numpy()
    out["nvfp4_f32/sf"] = u8(s)
    out["nvfp4_f32/ts"] = t.reshape(1).numpy()
    # 3D
    x3 = gen_bf16((3, 64, 128), 0.02, 10)
    p, s, t = Q.quantize_3d_to_nvfp4(x3)
    out["nvfp4_3d/x"] = bf16bits(x3)
    out["nvfp4_3d/packed"] = p.numpy()
    out["nvfp4_3d/sf"] = u8(s)
    out["nvfp4_3d/ts"] = bf16bits(t.reshape(1))

    # --- FP8 weight quant: every bf16 bit pattern as its own row ----------
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    q8, s8 = Q.quantize_2d_to_fp8(allbf.reshape(65536, 1))
    out["fp8_all/codes"] = u8(q8).reshape(-1)
    out["fp8_all/scale"] = bf16bits(s8).reshape(-1)
    x3 = gen_bf16((4, 32, 64), 0.02, 11)
    x3[1, 2] = 0.0
    q8, s8 = Q.quantize_3d_to_fp8(x3)
    out["fp8_3d/x"] = bf16bits(x3)
    out["fp8_3d/codes"] = u8(q8)
    out["fp8_3d/scale"] = bf16bits(s8)

    # --- FP8 activation quant, captured at the _scaled_mm call -----------
    from aeo_quant.bridges.gemma4.modeling import Gemma4TextExpertsFP8
    captured = {}

    def fake_scaled_mm(a, b, scale_a, scale_b, out_dtype):
        captured["a"] = a.clone()
        captured["sa"] = scale_a.clone()
        return torch.zeros(a.shape[0], b.shape[1], dtype=out_dtype)

    xa = gen_bf16((6, 64), 1.0, 12)
    xa[1] = 0.0
    xa[2] *= 1e-6
    xa[3, 7] = 5.0e4
    real = torch._scaled_mm
    torch._scaled_mm = fake_scaled_mm
    try:
        Gemma4TextExpertsFP8._fp8_linear(xa, torch.zeros(16, 64, dtype=torch.float8_e4m3fn),
                                        torch.ones(1, 16))
    finally:
        torch._scaled_mm = real
    out["fp8_act/x"] = bf16bits(xa)
    out["fp8_act/codes"] = u8(captured["a"])
    out["fp8_act/scale"] = captured["sa"].numpy().reshape(-1)

    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **out)

    # --- config-0 hashes --------------------------------------------------
    W = gen_bf16((1408, 2816), 0.02, 0)
    g = torch.Generator().manual_seed(0)
    _ = torch.randn(1408, 2816, generator=g)
    X = torch.randn(128, 2816, generator=g).to(torch.bfloat16)
    hashes = {"recipe": "g=torch.Generator().manual_seed(0); W=(randn(1408,2816,g)*0.02).bf16; "
                        "X=randn(128,2816,g).bf16 (same generator, drawn after W)"}
    for name, t in (("W", W), ("X", X)):
        p, s, ts = Q.quantize_2d_to_nvfp4(t)
        hashes[name] = {"input": sha(bf16bits(t)), "packed": sha(p.numpy()),
                        "sf": sha(u8(s)), "ts_bits": int(bf16bits(ts.reshape(1))[0])}
    with open(os.path.join(HERE, "config0_hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1)

    make_moe_golden(Q)


def _blockscaled_contract(a_packed, a_bs, a_ts, w_packed, w_bs, w_ts):
    """Published tl.dot_scaled contract on CPU: exact operands, float64 dot."""
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])

    def deq(p, s):
        nib = torch.stack([p >> 4, p & 0xF], -1).reshape(*p.shape[:-1], -1).long()
        v = lut[nib].reshape(*p.shape[:-1], -1, 16) * s.float().unsqueeze(-1)
        return v.reshape(*p.shape[:-1], -1).double()

    acc = (deq(a_packed, a_bs) @ deq(w_packed, w_bs).T).float()
    alpha = a_ts.float() * w_ts.float()
    return (acc * alpha).to(torch.bfloat16)


def make_moe_golden(Q):
    import aeo_quant.gpu.nvfp4_matmul as NM
    from aeo_quant.bridges.gemma4 import modeling as FM
    from aeo_quant.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4

    E, H, I, K = 8, 128, 64, 4
    cfg = types.SimpleNamespace(num_experts=E, hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")

    def gather(a_p, a_s, a_t, w_p, w_s, w_t, ids, *, out_dtype=torch.bfloat16):
        outs = []
        for j, e in enumerate(ids.tolist()):
            ap = a_p if a_p.ndim == 2 else a_p[j]
            asf = a_s if a_s.ndim == 2 else a_s[j]
            outs.append(_blockscaled_contract(ap, asf, a_t, w_p[e], w_s[e], w_t))
        return torch.stack(outs, 0)

    def prequant(a_p, a_s, a_t, w_p, w_s, w_t, *, out_dtype=torch.bfloat16):
        return _blockscaled_contract(a_p, a_s, a_t, w_p, w_s, w_t)

    NM.nvfp4_linear_3d_gather = gather
    NM.nvfp4_linear_prequantized = prequant   # nvfp4_linear looks this up at call time

    wgu = gen_bf16((E, 2 * I, H), 0.02, 20)
    wd = gen_bf16((E, H, I), 0.02, 21)
    m = Gemma4TextExpertsNVFP4(cfg)
    gp, gs, gt = Q.quantize_3d_to_nvfp4(wgu)
    dp, ds, dt = Q.quantize_3d_to_nvfp4(wd)
    m.gate_up_proj.copy_(gp); m.gate_up_proj_scale.copy_(gs)
    m.gate_up_proj_scale_2.copy_(gt.float())
    m.down_proj.copy_(dp); m.down_proj_scale.copy_(ds)
    m.down_proj_scale_2.copy_(dt.float())
    out = {"nv/gate_up_proj": gp.numpy(), "nv/gate_up_proj_scale": u8(gs),
           "nv/gate_up_proj_scale_2": np.array([float(gt)], np.float32),
           "nv/down_proj": dp.numpy(), "nv/down_proj_scale": u8(ds),
           "nv/down_proj_scale_2": np.array([float(dt)], np.float32)}

    g = torch.Generator().manual_seed(22)
    for T in (1, 7, 33):
        h = torch.randn(T, H, generator=g).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
        w = torch.softmax(torch.randn(T, K, generator=g), -1).to(torch.bfloat16)
        y = m.forward(h, idx, w)
        out[f"nv/T{T}/hidden"] = bf16bits(h)
        out[f"nv/T{T}/idx"] = idx.numpy().astype(np.int64)
        out[f"nv/T{T}/w"] = bf16bits(w)
        out[f"nv/T{T}/out"] = bf16bits(y)

    # FP8 experts with the _scaled_mm contract on CPU.
    def scaled_mm(a, b, scale_a, scale_b, out_dtype):
        acc = (a.float().double() @ b.float().double()).float()
        return ((acc * scale_a.float()) * scale_b.float()).to(out_dtype)

    fm = FM.Gemma4TextExpertsFP8(cfg)
    q1, s1 = Q.quantize_3d_to_fp8(wgu)
    q2, s2 = Q.quantize_3d_to_fp8(wd)
    fm.gate_up_proj.data = q1
    fm.down_proj.data = q2
    fm.gate_up_proj_scale = s1.squeeze(-1).unsqueeze(1).float().contiguous()
    fm.down_proj_scale = s2.squeeze(-1).unsqueeze(1).float().contiguous()
    out.update({"f8/gate_up_proj": u8(q1), "f8/gate_up_proj_scale": fm.gate_up_proj_scale.numpy(),
                "f8/down_proj": u8(q2), "f8/down_proj_scale": fm.down_proj_scale.numpy()})
    real = torch._scaled_mm
    torch._scaled_mm = scaled_mm
    try:
        for T in (1, 7, 33):
            h = torch.randn(T, H, generator=g).to(torch.bfloat16)
            idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
            w = torch.softmax(torch.randn(T, K, generator=g), -1).to(torch.bfloat16)
            y = fm.forward(h, idx, w)
            out[f"f8/T{T}/hidden"] = bf16bits(h)
            out[f"f8/T{T}/idx"] = idx.numpy().astype(np.int64)
            out[f"f8/T{T}/w"] = bf16bits(w)
            out[f"f8/T{T}/out"] = bf16bits(y)
    finally:
        torch._scaled_mm = real
    np.savez_compressed(os.path.join(HERE, "moe_golden.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the aeo-quant source tree>")
    main(sys.argv[1])
