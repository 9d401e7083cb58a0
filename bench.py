"""Benchmark: one-token NVFP4 MoE expert decode (Gemma-4 expert layer, batch 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

A step is one token through one Gemma-4-26B-A4B MoE layer: 128 NVFP4
experts (gate_up [1408, 2816], down [2816, 704]), top-8 routing, through
``Gemma4TextExpertsNVFP4.forward`` (the reference's class-swap module API).
Weights: bf16 N(0, 0.02) quantized on the device with the library's
quantizer; hidden bf16 N(0, 1); ids uniform without replacement; weights
softmax(N(0, 1)). 32 independent layers are resident and steps cycle through
them, so each step streams cold weights from HBM (26.8 MB per step, 830 MB
between revisits; L2 is 126 MB): inputs larger than L2, no flush needed.

The same line carries the other measured rows, each through the public API:
``prefill`` (the single NVFP4 linear at M = 128 with its HBM fraction, at
M = 8192 and 32768, and the grouped FP8 / NVFP4 expert prefill at 4096
tokens), ``decode_batch_sweep`` (batch 4, 16, 64 with an HBM roofline from
the realized unique experts), ``quantizer`` (NVFP4 activation quantization,
HBM GB/s) and ``ep`` (the expert-parallel stack of 4 layers over 65,536
Zipf-routed tokens on the same N GPUs, strong scaling, with the one-GPU time
of the same stack for the efficiency).

Multi-GPU: one-token decode does not shard (expert parallelism only pays at
prefill sizes), so N GPUs run N independent replicas; value = all ranks'
tokens / max-over-ranks device time ("scaling": "weak"). The ``ep`` leg is
the sharded workload.

``--impl reference`` times the reference algorithm on the host CPU: the
torch restatement in ``oracle/torch_port.py`` (the reference's own path needs
a GPU and Triton) on a bounded token sample with every host thread, rank 0
only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "aeo-quant_b200"))
sys.path.insert(0, ROOT)

E, H, I, TOPK = 128, 2816, 704, 8
EXPERT_BYTES = 1408 * 1408 + 1408 * 176 + 2816 * 352 + 2816 * 44  # packed + scales, 3,345,408
GATEUP_BYTES = 1408 * 1408 + 1408 * 176
DOWN_BYTES = 2816 * 352 + 2816 * 44
METRIC = "MoE decode tok/s (M=1 gather) + NVFP4 prefill TFLOPS, % of roofline"
FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum of one decode at this
# workload, from the committed ncu summary of each one-token kernel (None
# where the current kernel has not been captured).
NCU_TRAFFIC = {"stream": None, "tc": 27048448}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=320)
    p.add_argument("--warmup", type=int, default=32)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--no-prefill", action="store_true", help="skip the prefill GEMM measurements")
    p.add_argument("--no-ep", action="store_true", help="skip the expert-parallel (config 4) leg")
    p.add_argument("--workload", default="decode", choices=["decode", "ep", "gemm", "stack", "router", "grouped", "quant"],
                   help="decode: config 1 (default); ep: config 4, expert-parallel prefill stack; "
                        "gemm: config-0 NVFP4 linear at --gemm-m rows (profiling)")
    p.add_argument("--gemm-m", type=int, default=32768)
    p.add_argument("--tokens", type=int, default=32 * 2048, help="ep: tokens over all ranks")
    p.add_argument("--ep-layers", type=int, default=4)
    p.add_argument("--stack-layers", type=int, default=30, help="stack: decoder layers")
    p.add_argument("--prompt", type=int, default=2048, help="stack: prefill tokens")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.rows = []
        self.proc = None
        self.path = f"/tmp/aeoq_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if not self.proc:
            return
        time.sleep(0.2)
        self.proc.send_signal(2)
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            with open(self.path) as f:
                self.rows = [[c.strip() for c in line.split(",")] for line in f if line.strip()]
            os.remove(self.path)
        except Exception:
            self.rows = []

    def summary(self):
        rows = [r for r in self.rows if len(r) > 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def make_layers(torch, L, device, seed=0):
    from aeo_quant_b200.gpu import quant as Q
    layers = []
    for li in range(L):
        g = torch.Generator(device=device).manual_seed(seed * 1000 + li)
        w = torch.randn(E, 2 * I, H, generator=g, device=device, dtype=torch.bfloat16).mul_(0.02)
        gp, gs, gt = Q.quantize_3d_to_nvfp4(w)
        del w
        w = torch.randn(E, H, I, generator=g, device=device, dtype=torch.bfloat16).mul_(0.02)
        dp, ds, dt = Q.quantize_3d_to_nvfp4(w)
        del w
        layers.append((gp, gs, gt.float(), dp, ds, dt.float()))
    torch.cuda.synchronize()
    return layers


def make_module(torch, device, layer):
    import types
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    cfg = types.SimpleNamespace(num_experts=E, hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")
    m = Gemma4TextExpertsNVFP4(cfg)
    gp, gs, gt, dp, ds, dt = layer
    # buffers alias the resident layer tensors (no copies)
    m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2 = gp, gs, gt
    m.down_proj, m.down_proj_scale, m.down_proj_scale_2 = dp, ds, dt
    return m


def routing(torch, S, B, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.stack([torch.randperm(E, generator=g)[:TOPK] for _ in range(B)]) for _ in range(S)])
    w = torch.softmax(torch.randn(S, B, TOPK, generator=g), -1).to(torch.bfloat16)
    h = torch.randn(S, B, H, generator=g).to(torch.bfloat16)
    return idx, w, h


def decode_config(B, L, world):
    """The ``config`` object of the decode line, shared by both arms."""
    return {"workload": f"config1: M=1 NVFP4 expert-gather decode, one MoE layer, batch {B}",
            "experts": E, "hidden": H, "intermediate": I, "top_k": TOPK, "batch": B,
            "resident_layers": L, "l2": f"inputs larger than L2: {L} layers cycled, "
            f"{L * 428} MB resident, 26.8 MB streamed per step",
            "parallelism": f"replicas x{world}", "timing": "one CUDA graph of K steps, CUDA events"}


def cpu_baseline(seconds, batch=1):
    """Time the reference's CPU arithmetic for the decode on the host: the
    torch restatement in ``oracle/torch_port.py`` (quantize the hidden
    vector, dequantize the 8 routed experts' NVFP4 weights to f32, f32
    matmuls, every bf16 rounding of ``_forward_decode_3d``), one process
    using every host thread, over a 128-expert layer of random packed
    weights (the time per token does not depend on the values). Tokens run
    back to back for about ``seconds``; value = tokens / elapsed."""
    import torch
    from oracle import torch_port as TP
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(7)
    gu = torch.randint(0, 256, (E, 2 * I, H // 2), generator=g, dtype=torch.uint8)
    dw = torch.randint(0, 256, (E, H, I // 2), generator=g, dtype=torch.uint8)
    # e4m3 block scales 0x20..0x3f (2^-3 .. ~0.94): finite, no NaN codes
    gs = torch.randint(0x20, 0x40, (E, 2 * I, H // 16), generator=g, dtype=torch.uint8)
    ds = torch.randint(0x20, 0x40, (E, H, I // 16), generator=g, dtype=torch.uint8)
    m = TP.Experts(gu, gs, 1e-3, dw, ds, 1e-3)

    def one(i):
        gi = torch.Generator().manual_seed(100 + i)
        h = torch.randn(batch, H, generator=gi).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(E, generator=gi)[:TOPK] for _ in range(batch)])
        w = torch.softmax(torch.randn(batch, TOPK, generator=gi), -1).to(torch.bfloat16)
        TP.forward(m, h, idx, w)

    one(0)   # warm-up
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or done < 3:
        one(done + 1)
        done += 1
    dt_s = time.perf_counter() - t0
    return {"value": done * batch / dt_s, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{done} steps of batch {batch} x 1 layer (128 experts, top-8) through the torch "
                      f"restatement of the reference forward (oracle/torch_port.py: NVFP4 dequantize + f32 "
                      f"matmul), one process, torch threads {threads}, {dt_s:.1f} s"}


def run_reference(args, rank):
    if rank != 0:
        return
    t_budget = max(5.0, min(30.0, args.steps * 0.5))
    cb = cpu_baseline(t_budget, args.batch)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * args.batch / cb["value"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp4(e2m1)+e4m3 scales, fp32 accumulate, bf16 io", "data": "synthetic",
        "config": decode_config(args.batch, args.layers, args.gpus),
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _graph_time_us(torch, dev, fn, iters):
    """Mean device time of fn over one CUDA graph of `iters` calls (after warm-up)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    sg = torch.cuda.Stream(dev)
    sg.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(sg):
        fn()
        with torch.cuda.graph(g, stream=sg):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream(dev).wait_stream(sg)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / iters


def measure_prefill(torch, dev, lib, A):
    """Config 0 (NVFP4 linear N=1408, K=2816) at M = 128 and at prefill sizes,
    and the config-2 FP8 expert prefill (4096 tokens, top-8), through the
    public API, as CUDA-graph replays. FP4/FP8 fractions are of the nominal
    dense peaks (9 / 4.5 PFLOP/s): no measured FP4/FP8 peak exists."""
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    from aeo_quant_b200.gpu import nvfp4_matmul as NM
    from aeo_quant_b200.gpu import quant as Q
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(1408, 2816, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wp, wsf, wts = Q.quantize_2d_to_nvfp4(w)
    wts = wts.float()
    out = {}
    for M in (128, 8192, 32768):
        x = torch.randn(M, 2816, generator=g, device=dev).to(torch.bfloat16)
        ap, asf, ats = Q.quantize_2d_to_nvfp4(x)
        us = _graph_time_us(torch, dev, lambda: NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts),
                            20 if M < 32768 else 10)
        tf = 2.0 * M * 1408 * 2816 / us / 1e6
        out[f"config0_M{M}"] = {"us": round(us, 2), "tflops": round(tf, 1), "frac_fp4_nominal": round(tf / 9000, 4)}
        if M == 128:
            # HBM-bound shape: packed operands + scales in, bf16 out
            byt = M * 2816 * 0.5625 + 1408 * 2816 * 0.5625 + M * 1408 * 2
            gbs = byt / (us * 1e-6) / 1e9
            out[f"config0_M{M}"].update({"algorithmic_bytes": int(byt), "gbs": round(gbs, 1),
                                         "frac_hbm": round(gbs / peaks()[0], 4)})
    T, k = 4096, TOPK
    gq, gs = Q.quantize_3d_to_fp8((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    dq, ds = Q.quantize_3d_to_fp8((torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    gsb, dsb = gs.reshape(-1).float().contiguous(), ds.reshape(-1).float().contiguous()
    h = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev)
    wv, ids = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    wts8 = (wv / wv.sum(-1, keepdim=True)).to(torch.bfloat16)
    us = _graph_time_us(torch, dev, lambda: moe_ops.fp8_experts_grouped(h, ids, wts8, gq, gsb, dq, dsb), 5)
    tf = T * k * 11894784 / us / 1e6
    out["config2_fp8_T4096"] = {"us": round(us, 1), "tflops": round(tf, 1), "frac_fp8_nominal": round(tf / 4500, 4)}
    del gq, dq
    gp, gsf, gt = Q.quantize_3d_to_nvfp4((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    dp, dsf, dt = Q.quantize_3d_to_nvfp4((torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    us = _graph_time_us(torch, dev, lambda: moe_ops.nvfp4_experts_grouped(h, ids, wts8, gp, gsf, gt.float(), dp, dsf,
                                                                          dt.float()), 5)
    tf = T * k * 11894784 / us / 1e6
    out["config2_shapes_nvfp4_T4096"] = {"us": round(us, 1), "tflops": round(tf, 1),
                                         "frac_fp4_nominal": round(tf / 9000, 4)}
    return out


def main_gemm(args, local):
    """Config-0 weights (N=1408, K=2816) against --gemm-m activation rows
    through nvfp4_linear_prequantized: W warm-up calls, then K timed calls
    (CUDA events). Used for the GEMM profiles."""
    import torch
    from aeo_quant_b200.gpu import nvfp4_matmul as NM
    from aeo_quant_b200.gpu import quant as Q
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(1408, 2816, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wp, wsf, wts = Q.quantize_2d_to_nvfp4(w)
    wts = wts.float()
    M = args.gemm_m
    x = torch.randn(M, 2816, generator=g, device=dev).to(torch.bfloat16)
    ap, asf, ats = Q.quantize_2d_to_nvfp4(x)
    for _ in range(max(3, args.warmup)):
        NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        NM.nvfp4_linear_prequantized(ap, asf, ats, wp, wsf, wts)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / args.steps
    tf = 2.0 * M * 1408 * 2816 / us / 1e6
    print(json.dumps({"metric": "NVFP4 prefill TFLOPS (config-0 shapes)", "value": round(tf, 1), "unit": "TFLOP/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1000.0,
                      "higher_is_better": True, "config": {"workload": f"config0 GEMM M={M} N=1408 K=2816"},
                      "frac_fp4_nominal": round(tf / 9000, 4)}), flush=True)


def main_grouped(args, local):
    """The grouped expert forwards alone at the FP8 prefill shapes (128
    experts, H 2816, I 704, --tokens tokens, softmax top-8): FP8 and NVFP4,
    each W warm-up calls then K calls timed with CUDA events. Used for the
    launch lists and captures of the grouped pipeline."""
    import torch
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    from aeo_quant_b200.gpu import quant as Q
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(0)
    T = args.tokens
    h = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    wv, ids = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device=dev), -1), TOPK, dim=-1)
    wts = (wv / wv.sum(-1, keepdim=True)).to(torch.bfloat16)
    out = {}
    gq, gs = Q.quantize_3d_to_fp8((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    dq, ds = Q.quantize_3d_to_fp8((torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    gsb, dsb = gs.reshape(-1).float().contiguous(), ds.reshape(-1).float().contiguous()
    gp, gsf, gt = Q.quantize_3d_to_nvfp4((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    dp, dsf, dt = Q.quantize_3d_to_nvfp4((torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    gt, dt = gt.float(), dt.float()
    for name, fn in (("fp8", lambda: moe_ops.fp8_experts_grouped(h, ids, wts, gq, gsb, dq, dsb)),
                     ("nvfp4", lambda: moe_ops.nvfp4_experts_grouped(h, ids, wts, gp, gsf, gt, dp, dsf, dt))):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / args.steps
        out[name] = {"us": round(us, 1), "tflops": round(T * TOPK * 11894784 / us / 1e6, 1)}
    print(json.dumps({"metric": "grouped expert forward", "config": {"workload": f"{T} tokens, top-8, 128 experts"},
                      **out}), flush=True)


def ep_layers(torch, dev, rank, world, n_layers, owner):
    """The config-4 stack's NVFP4 expert layers for this rank: expert e of
    layer l drawn from its own seeded generator (the same weights whatever
    the world size or placement), this rank's experts (owner[e] == rank,
    ascending id; all of them when owner is None) quantized on the device."""
    import types
    from aeo_quant_b200.bridges.gemma4.expert_parallel import ExpertParallelNVFP4
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    from aeo_quant_b200.gpu import quant as Q
    mine = list(range(E)) if owner is None else [e for e in range(E) if int(owner[e]) == rank]
    cfg = types.SimpleNamespace(num_experts=len(mine), hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")
    layers = []
    for l in range(n_layers):
        wgu = torch.empty(len(mine), 2 * I, H, dtype=torch.bfloat16, device=dev)
        wd = torch.empty(len(mine), H, I, dtype=torch.bfloat16, device=dev)
        for i, e in enumerate(mine):
            ge = torch.Generator(device=dev).manual_seed(100000 * (l + 1) + e)
            wgu[i] = (torch.randn(2 * I, H, generator=ge, device=dev) * 0.02).to(torch.bfloat16)
            wd[i] = (torch.randn(H, I, generator=ge, device=dev) * 0.02).to(torch.bfloat16)
        m = Gemma4TextExpertsNVFP4(cfg).to(dev)
        gp, gs, gt = Q.quantize_3d_to_nvfp4(wgu)
        dp, ds, dt = Q.quantize_3d_to_nvfp4(wd)
        del wgu, wd
        m.gate_up_proj.copy_(gp); m.gate_up_proj_scale.copy_(gs); m.gate_up_proj_scale_2.copy_(gt.float())
        m.down_proj.copy_(dp); m.down_proj_scale.copy_(ds); m.down_proj_scale_2.copy_(dt.float())
        layers.append(ExpertParallelNVFP4(m, E, owner=owner, equal_tokens=True) if owner is not None else m)
    return layers


def zipf_ids(torch, dev, T, seed):
    """Zipf(s=1.2) over a seeded permutation of the experts, 8 distinct per
    token; softmax(N(0,1)) weights."""
    g = torch.Generator(device=dev).manual_seed(seed)
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(5)).to(dev)
    p = 1.0 / torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** 1.2
    ids = perm[torch.multinomial(p.expand(T, E), TOPK, replacement=False, generator=g)]
    wts = torch.softmax(torch.randn(T, TOPK, generator=g, device=dev), -1).to(torch.bfloat16)
    return ids, wts


def run_ep(args, rank, world, local, steps, warmup):
    """Config 4: a stack of ``--ep-layers`` NVFP4 MoE layers (128 experts,
    H 2816, I 704) over ``--tokens`` tokens split by sequence over the
    ranks, Zipf(1.2) top-8 routing. With N > 1 experts are placed on ranks by
    ``balanced_placement`` of the global routing histogram (E/N per rank);
    dispatch (NVFP4-packed rows) and combine (bf16 rows) are NCCL
    all-to-alls. One step = the whole stack over every rank's tokens; value
    = tokens / max-over-ranks device time (strong scaling: the token count
    is fixed). At N = 1 it is the one-GPU forward. The process group must be
    initialised when N > 1. Returns the leg's dict on rank 0."""
    import torch
    import torch.distributed as dist
    from aeo_quant_b200.bridges.gemma4.expert_parallel import balanced_placement
    dev = torch.device("cuda", local)
    T = args.tokens // world
    ids, wts = zipf_ids(torch, dev, T, 1000 + rank)
    hid = torch.randn(T, H, generator=torch.Generator(device=dev).manual_seed(2000 + rank), device=dev).to(
        torch.bfloat16)
    owner = None
    if world > 1:
        load = torch.bincount(ids.reshape(-1), minlength=E).to(torch.float64)
        dist.all_reduce(load)
        owner = balanced_placement(load.cpu(), world)
    layers = ep_layers(torch, dev, rank, world, args.ep_layers, owner)

    def step(x):
        for lay in layers:
            x = lay(x, ids, wts)
        return x

    def timed(fn, K):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(warmup):
        step(hid)
    with ClockSampler(local) as clk:
        ms = timed(lambda: step(hid), steps)
    phases = None
    if world > 1:
        # phase split: CUDA events at each phase start (device-timeline gaps,
        # so idle time waiting on the host counts in the phase it delays);
        # the per-phase median of three instrumented steps
        runs = []
        for _ in range(3):
            evs = []

            def mark(name, evs=evs):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                evs.append((name, ev))
            for lay in layers:
                lay.mark = mark
            step(hid)
            torch.cuda.synchronize()
            for lay in layers:
                lay.mark = None
            acc = {"dispatch": 0.0, "experts": 0.0, "combine": 0.0}
            for (n0, a), (_, b) in zip(evs, evs[1:]):
                if n0 in acc:
                    acc[n0] += a.elapsed_time(b)
            runs.append([acc["dispatch"], acc["experts"], acc["combine"]])
        ph = torch.tensor(runs, device=dev).median(dim=0).values
        dist.all_reduce(ph, op=dist.ReduceOp.MAX)
        phases = dict(zip(("dispatch", "experts", "combine"), [round(v, 3) for v in ph.tolist()]))
    # e2e: this rank's tokens from pinned host memory, the output back
    hid_h = hid.cpu().pin_memory()
    out_h = torch.empty_like(hid_h).pin_memory()
    x_in = torch.empty_like(hid)

    def e2e_step():
        x_in.copy_(hid_h, non_blocking=True)
        out_h.copy_(step(x_in), non_blocking=True)
    ms_e2e = timed(e2e_step, steps)
    # the same stack with every expert on one GPU, for the efficiency
    ms_1 = None
    if world > 1:
        del layers
        torch.cuda.empty_cache()
        if rank == 0:
            parts = [zipf_ids(torch, dev, T, 1000 + r) for r in range(world)]
            all_ids = torch.cat([p[0] for p in parts])
            all_w = torch.cat([p[1] for p in parts])
            all_h = torch.cat([torch.randn(T, H, generator=torch.Generator(device=dev).manual_seed(2000 + r),
                                           device=dev).to(torch.bfloat16) for r in range(world)])
            one = ep_layers(torch, dev, 0, 1, args.ep_layers, None)

            def step1():
                x = all_h
                for lay in one:
                    x = lay(x, all_ids, all_w)
            for _ in range(warmup):
                step1()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                step1()
            e1.record()
            torch.cuda.synchronize()
            ms_1 = e0.elapsed_time(e1)
            del one
        dist.barrier()
    if rank != 0:
        return None
    flops = args.tokens * TOPK * 11894784 * args.ep_layers * steps
    ach = flops / (ms / 1000.0) / 1e12 / world
    out = {"workload": f"config4: NVFP4 MoE stack, {args.ep_layers} layers, {args.tokens} tokens "
                       f"(Zipf(1.2) top-8) over {world} GPU(s)",
           "tok_s": round(args.tokens * steps / (ms / 1000.0), 1), "ms_per_step": round(ms / steps, 3),
           "steps": steps, "warmup": warmup, "scaling": "strong",
           "placement": "balanced_placement of the global routing histogram" if world > 1 else "one GPU, all experts",
           "phase_ms_per_step": phases,
           "tflops_per_gpu": round(ach, 1), "frac_fp4_nominal": round(ach / 9000.0, 4),
           "e2e_tok_s": round(args.tokens * steps / (ms_e2e / 1000.0), 1),
           "clocks": clk.summary()}
    if ms_1 is not None:
        out["one_gpu_ms_per_step"] = round(ms_1 / steps, 3)
        out["efficiency_vs_one_gpu"] = round(ms_1 / (world * ms), 4)
    return out


def main_ep(args, rank, world, local):
    """``--workload ep``: the config-4 leg alone, as its own JSON line."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    r = run_ep(args, rank, world, local, args.steps, max(3, args.warmup))
    if rank == 0:
        print(json.dumps({"metric": "config4 expert-parallel MoE stack tok/s", "value": r["tok_s"], "unit": "tok/s",
                          "n_gpus": world, "higher_is_better": True, "ep": r}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def stack_config(layers):
    """Config 3: a Gemma-4-26B-A4B-shaped text decoder. Pinned: hidden 2816,
    128 experts top-8, expert intermediate 704, vocab 262144, 30 layers with
    a sliding window of 1024 on 5 of every 6. Chosen (the real config.json
    is not available): 16 query heads and 8 KV heads of 256 (512 on
    full-attention layers), dense MLP 2112, no per-layer input embedding."""
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    types_ = [("full_attention" if (i + 1) % 6 == 0 else "sliding_attention") for i in range(layers)]
    return Gemma4TextConfig(
        hidden_size=H, num_hidden_layers=layers, num_attention_heads=16, num_key_value_heads=8, head_dim=256,
        global_head_dim=512, intermediate_size=2112, moe_intermediate_size=I, num_experts=E, top_k_experts=TOPK,
        enable_moe_block=True, vocab_size=262144, vocab_size_per_layer_input=262144,
        hidden_size_per_layer_input=0, sliding_window=1024, layer_types=types_, max_position_embeddings=8192)


def _our_kernel_launches(torch, fn):
    """Kernels of this library launched by one call of ``fn`` (profiler
    pass outside any timed region); None if the profiler is unavailable."""
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        n = 0
        for ev in prof.events():
            name = ev.name or ""
            if ev.device_type == torch.autograd.DeviceType.CUDA and ("aeoq::" in name or "dtc::" in name):
                n += 1
        return n
    except Exception:
        return None


def main_router(args, local):
    """The Gemma-4 router alone (config-3 shapes: H 2816, 128 experts,
    top-8): the fused kernel and HF's eager forward, one token and
    ``--prompt`` tokens, each timed as one CUDA graph of repeated calls."""
    import torch
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextRouter
    from aeo_quant_b200.bridges.gemma4.loader import swap_routers

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    r = Gemma4TextRouter(stack_config(6)).to(device=dev, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        r.proj.weight.normal_(0.0, 0.5)
    swap_routers(torch.nn.Sequential(r))
    from aeo_quant_b200.bridges.gemma4 import router as R
    out = {}
    with torch.no_grad():
        for T in (1, 16, 64, 128, 256, 512, args.prompt):
            x = torch.randn(T, H, device=dev).to(torch.bfloat16)
            n = 200 if T <= 64 else 50
            old, R.FUSED_MAX_TOKENS = R.FUSED_MAX_TOKENS, 1 << 30     # the fused kernel at every size
            out[f"fused_kernel_T{T}_us"] = round(_graph_time_us(torch, dev, lambda: r(x), n), 2)
            R.FUSED_MAX_TOKENS = old
            out[f"module_T{T}_us"] = round(_graph_time_us(torch, dev, lambda: r(x), n), 2)
            out[f"hf_eager_T{T}_us"] = round(
                _graph_time_us(torch, dev, lambda: Gemma4TextRouter.forward(r, x), n), 2)
    print(json.dumps({"metric": "Gemma-4 router latency", "unit": "us", "higher_is_better": False,
                      "config": {"workload": "router alone, H 2816, 128 experts, top-8, bf16"}, **out}), flush=True)


def main_stack(args, local):
    """Config 3: random-init Gemma-4-shaped stack, experts converted to NVFP4
    on the GPU and run through the swapped ``Gemma4TextExpertsNVFP4``; HF
    transformers (eager PyTorch) for everything else. Prefill 2048 tokens,
    then K greedy decode steps, batch 1. value = decode tok/s."""
    import torch
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    from aeo_quant_b200.bridges.gemma4.loader import quantize_experts_to_nvfp4

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, P, K, W = args.stack_layers, args.prompt, args.steps, max(3, args.warmup)
    torch.manual_seed(0)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = Gemma4ForCausalLM(stack_config(L)).eval()
    torch.set_default_dtype(old)
    n_conv = quantize_experts_to_nvfp4(model)
    torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(10, 262144, (1, P), generator=g).to(dev)

    def prefill():
        out = model(ids, use_cache=True)
        return out.past_key_values, out.logits[:, -1:].argmax(-1)

    def decode(pkv, nxt, n):
        for _ in range(n):
            out = model(nxt, past_key_values=pkv, use_cache=True)
            pkv, nxt = out.past_key_values, out.logits[:, -1:].argmax(-1)
        return pkv, nxt

    from aeo_quant_b200.bridges.gemma4.loader import swap_routers

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def timed(clk_holder):
        """Warm-up, then one timed prefill and K timed decode steps."""
        pkv, nxt = prefill()
        decode(pkv, nxt, W)
        del pkv
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ev[0].record()
            pkv, nxt = prefill()
            ev[1].record()
            ev[2].record()
            pkv, nxt = decode(pkv, nxt, K)
            ev[3].record()
            torch.cuda.synchronize()
        clk_holder.append(clk.summary())
        return ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3]), pkv, nxt

    clocks = []
    with torch.no_grad():
        # experts swapped, HF's eager router
        t_pre_x, t_dec_x, _, _ = timed(clocks)
        # experts and router swapped (the product configuration)
        n_routers = swap_routers(model)
        t_pre, t_dec, pkv, nxt = timed(clocks)
        n_dec = _our_kernel_launches(torch, lambda: decode(pkv, nxt, 1))
        # router alone, one token and the prefill's tokens
        lay = model.model.layers[0]
        xr1 = torch.randn(1, H, device=dev).to(torch.bfloat16)
        xrp = torch.randn(P, H, device=dev).to(torch.bfloat16)
        from transformers.models.gemma4.modeling_gemma4 import Gemma4TextRouter
        router_us = {
            "fused_T1": round(_graph_time_us(torch, dev, lambda: lay.router(xr1), 200), 2),
            "hf_eager_T1": round(_graph_time_us(torch, dev, lambda: Gemma4TextRouter.forward(lay.router, xr1), 200), 2),
            f"fused_T{P}": round(_graph_time_us(torch, dev, lambda: lay.router(xrp), 50), 2),
            f"hf_eager_T{P}": round(_graph_time_us(torch, dev, lambda: Gemma4TextRouter.forward(lay.router, xrp), 50), 2),
        }
        # e2e: each step's token id goes up from pinned host memory and the
        # greedy token comes back before the next step is issued
        tok_h = torch.empty(1, 1, dtype=torch.int64).pin_memory()
        tok_h.copy_(nxt.cpu())
        x = torch.empty(1, 1, dtype=torch.int64, device=dev)
        pkv2, _ = prefill()
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(K):
            x.copy_(tok_h, non_blocking=True)
            out = model(x, past_key_values=pkv2, use_cache=True)
            pkv2 = out.past_key_values
            tok_h.copy_(out.logits[:, -1:].argmax(-1), non_blocking=True)
            torch.cuda.current_stream().synchronize()
        ev[1].record()
        torch.cuda.synchronize()
        t_e2e = ev[0].elapsed_time(ev[1])
    value = K / (t_dec / 1000.0)
    print(json.dumps({
        "metric": "Gemma-4 stack greedy decode tok/s (batch 1)", "value": round(value, 2), "unit": "tok/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": t_dec / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "NVFP4 experts (fp32 accumulate), bf16 elsewhere",
        "data": "synthetic (random-init weights N(0,0.02), experts quantized to NVFP4 on device; random prompt)",
        "config": {"workload": f"config3: random-init Gemma-4-26B-A4B-shaped stack, {L} layers, "
                               f"prefill {P} tokens then {K} greedy decode steps, batch 1",
                   "experts_converted": n_conv, "routers_swapped": n_routers, "hidden": H, "experts": E, "top_k": TOPK, "intermediate": I,
                   "non_expert": "HF transformers eager (attention, dense MLP, lm_head)",
                   "l2": "inputs larger than L2 (12.8 GB of expert weights per decode step)",
                   "timing": "CUDA events around the prefill and around K decode steps"},
        "prefill": {"tokens": P, "ms": round(t_pre, 3), "tok_s": round(P / (t_pre / 1000.0), 1)},
        "experts_only_swap": {"decode_tok_s": round(K / (t_dec_x / 1000.0), 2), "prefill_ms": round(t_pre_x, 3),
                              "note": "HF eager router in front of the swapped experts"},
        "router_us": router_us,
        "gpu_launches": None if n_dec is None else n_dec * K,
        "gpu_launches_per_decode_step": n_dec,
        "clocks": clocks[-1],
        "e2e": {"value": round(K / (t_e2e / 1000.0), 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8, "path": "model forward per token, token id from pinned host, "
                                                 "greedy token read back each step"},
    }), flush=True)


def measure_batch_sweep(torch, dev, mods, L, steps, seed):
    """Config 1 at batch 4, 16 and 64: B tokens through one MoE layer via
    the module API (the reference's prefill semantics for B > 1), layers
    cycled as in the headline, timed as one CUDA graph of ``steps`` calls.
    HBM roofline per B with the realized unique experts U per step:
    bytes = U * 3,345,408 + B * 2816 * 4 + B * 8 * 10."""
    hbm = peaks()[0]
    out = {}
    for B in (4, 16, 64):
        S = steps + 4
        idx, wts, hid = routing(torch, S, B, seed + B)
        idx_d, wts_d, hid_d = idx.to(dev), wts.to(dev), hid.to(dev)
        uniq = sum(len(set(idx[s2].reshape(-1).tolist())) for s2 in range(4, S)) / steps
        for s2 in range(4):
            mods[s2 % L](hid_d[s2], idx_d[s2], wts_d[s2])
        torch.cuda.synchronize()
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                for s2 in range(4, S):
                    mods[s2 % L](hid_d[s2], idx_d[s2], wts_d[s2])
        torch.cuda.current_stream(dev).wait_stream(cs)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / steps
        byt = uniq * EXPERT_BYTES + B * H * 4 + B * TOPK * 10
        gbs = byt / (us * 1e-6) / 1e9
        out[f"B{B}"] = {"us_per_step": round(us, 2), "tok_s": round(B / (us * 1e-6), 1),
                        "unique_experts": round(uniq, 2), "algorithmic_bytes": int(byt), "gbs": round(gbs, 1),
                        "frac_hbm": round(gbs / hbm, 4)}
        del g
    return out


def measure_quantizer(torch, dev):
    """The NVFP4 activation quantizer (quantize_2d_to_nvfp4) on 32768 x 2816
    bf16 (184.5 MB, larger than L2), through the public API, one CUDA graph
    of 10 calls. Algorithmic bytes per element: 2 read + 0.5625 written (the
    amax pass's second read is not counted)."""
    from aeo_quant_b200.gpu import quant as Q
    x = torch.randn(32768, H, generator=torch.Generator(device=dev).manual_seed(3), device=dev).to(torch.bfloat16)
    us = _graph_time_us(torch, dev, lambda: Q.quantize_2d_to_nvfp4(x), 10)
    byt = x.numel() * 2.5625
    gbs = byt / (us * 1e-6) / 1e9
    return {"shape": [32768, H], "us": round(us, 2), "algorithmic_bytes": int(byt), "gbs": round(gbs, 1),
            "frac_hbm": round(gbs / peaks()[0], 4)}


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "ep":
        main_ep(args, rank, world, local)
        return
    if args.workload == "gemm":
        main_gemm(args, local)
        return
    if args.workload == "grouped":
        main_grouped(args, local)
        return
    if args.workload == "quant":
        import torch
        torch.cuda.set_device(local)
        print(json.dumps({"metric": "NVFP4 activation quantizer", "quantizer":
                          measure_quantizer(torch, torch.device("cuda", local))}), flush=True)
        return
    if args.workload == "stack":
        main_stack(args, local)
        return
    if args.workload == "router":
        main_router(args, local)
        return
    import torch
    import torch.distributed as dist
    from aeo_quant_b200 import _capi as A
    from aeo_quant_b200.bridges.gemma4 import moe_ops

    if world > 1:
        dist.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, K, W = args.batch, args.steps, max(3, args.warmup)
    L = args.layers

    layers = make_layers(torch, L, dev, seed=rank + 1)
    mods = [make_module(torch, dev, lay) for lay in layers]
    S = K + W
    idx, wts, hid = routing(torch, S, B, 11 + rank)
    idx_d, wts_d, hid_d = idx.to(dev), wts.to(dev), hid.to(dev)

    def step(s):
        return mods[s % L](hid_d[s], idx_d[s], wts_d[s])

    # warm-up (eager, public API)
    for s in range(W):
        step(s)
    torch.cuda.synchronize()

    # capture the K timed steps in one CUDA graph (launch overhead out of the
    # device timeline; every step still launches its own kernels)
    cs = torch.cuda.Stream(dev)
    cs.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cs):
        step(W)
        with torch.cuda.graph(graph, stream=cs):
            outs = [step(W + s) for s in range(K)]
    torch.cuda.current_stream(dev).wait_stream(cs)
    torch.cuda.synchronize()
    graph.replay()   # warm replay
    torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        cur = torch.cuda.current_stream(dev)
        ev0.record(cur)
        graph.replay()
        ev1.record(cur)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * B * K / (ms_max / 1000.0)

    # ---- per-kernel timing for the roofline (same stream, CUDA events) ----
    lib = A.load()
    out = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    fws_n = lib.aeoq_moe_nvfp4_decode_fused_workspace_size(TOPK, H, I)
    fws = torch.zeros(fws_n, dtype=torch.uint8, device=dev)
    uws_n = lib.aeoq_moe_nvfp4_decode_workspace_size(TOPK, H, I)
    uws = torch.empty(uws_n, dtype=torch.uint8, device=dev)

    tws_n = lib.aeoq_moe_nvfp4_decode_tc_workspace_size(TOPK, H, I)
    tws = torch.zeros(max(tws_n, 1), dtype=torch.uint8, device=dev)
    sws_n = lib.aeoq_moe_nvfp4_decode_stream_workspace_size(TOPK, H, I)
    sws = torch.zeros(max(sws_n, 1), dtype=torch.uint8, device=dev)
    err = A.err_word(dev)

    def launch(fn, s, ws, ws_n):
        gp, gs, gt, dp, ds, dt = layers[s % L]
        extra = (err.data_ptr(),) if fn in (lib.aeoq_moe_nvfp4_decode_tc, lib.aeoq_moe_nvfp4_decode_stream) else ()
        return fn(hid_d[s].data_ptr(), idx_d[s].data_ptr(), A.I64, wts_d[s].data_ptr(), TOPK,
                  gp.data_ptr(), gs.data_ptr(), gt.data_ptr(), A.F32, dp.data_ptr(), ds.data_ptr(),
                  dt.data_ptr(), A.F32, E, H, I, out.data_ptr(), ws.data_ptr(), ws_n, *extra,
                  torch.cuda.current_stream(dev).cuda_stream)

    def time_graph(fn, ws, ws_n):
        sg = torch.cuda.Stream(dev)
        sg.wait_stream(torch.cuda.current_stream(dev))
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.stream(sg):
            for s in range(3):
                A.check(launch(fn, s, ws, ws_n))
            with torch.cuda.graph(g2, stream=sg):
                for s in range(K):
                    A.check(launch(fn, W + s, ws, ws_n))
        torch.cuda.current_stream(dev).wait_stream(sg)
        torch.cuda.synchronize()
        g2.replay()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        g2.replay()
        a1.record()
        torch.cuda.synchronize()
        return a0.elapsed_time(a1) / K

    stage_ms = {}
    tc_path = B == 1 and moe_ops.DECODE_PATH in ("auto", "tc") and bool(
        lib.aeoq_moe_nvfp4_decode_tc_supported(TOPK, H, I))
    stream_path = B == 1 and bool(lib.aeoq_moe_nvfp4_decode_stream_supported(TOPK, H, I))
    if B == 1:
        if stream_path:
            stage_ms["stream"] = time_graph(lib.aeoq_moe_nvfp4_decode_stream, sws, sws_n)
        if tc_path:
            stage_ms["tc"] = time_graph(lib.aeoq_moe_nvfp4_decode_tc, tws, tws_n)
        stage_ms["fused"] = time_graph(lib.aeoq_moe_nvfp4_decode_fused, fws, fws_n)
        stage_ms["unfused"] = time_graph(lib.aeoq_moe_nvfp4_decode, uws, uws_n)

    # ---- prefill: config-0 GEMMs and the config-2 FP8 expert prefill ----
    prefill = measure_prefill(torch, dev, lib, A) if (B == 1 and not args.no_prefill) else None
    sweep = measure_batch_sweep(torch, dev, mods, L, min(K, 20), 31 + rank) if (
        B == 1 and not args.no_prefill) else None
    quantizer = measure_quantizer(torch, dev) if (B == 1 and not args.no_prefill) else None

    # ---- end to end through the public module API with host buffers ----
    # Each step's inputs (hidden, ids, weights) sit in one pinned host row and
    # go up in one copy; the output comes back with one copy and a sync.
    nb_h, nb_i, nb_w = B * H * 2, B * TOPK * 8, B * TOPK * 2
    stage_h = torch.empty(S, nb_h + nb_i + nb_w, dtype=torch.uint8).pin_memory()
    stage_h[:, :nb_h].copy_(hid.reshape(S, -1).view(torch.uint8))
    stage_h[:, nb_h:nb_h + nb_i].copy_(idx.reshape(S, -1).contiguous().view(torch.uint8))
    stage_h[:, nb_h + nb_i:].copy_(wts.reshape(S, -1).contiguous().view(torch.uint8))
    stage_d = torch.empty(nb_h + nb_i + nb_w, dtype=torch.uint8, device=dev)
    h_in = stage_d[:nb_h].view(torch.bfloat16).view(B, H)
    i_in = stage_d[nb_h:nb_h + nb_i].view(torch.int64).view(B, TOPK)
    w_in = stage_d[nb_h + nb_i:].view(torch.bfloat16).view(B, TOPK)
    out_h = torch.empty(B, H, dtype=torch.bfloat16).pin_memory()
    n_e2e = min(K, 200)

    def e2e_step(s):
        stage_d.copy_(stage_h[s], non_blocking=True)
        y = mods[s % L](h_in, i_in, w_in)
        out_h.copy_(y, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for s in range(W):
        e2e_step(s)
    if world > 1:
        dist.barrier()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for s in range(n_e2e):
        e2e_step(W + s)
    b1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([b0.elapsed_time(b1)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_val = world * B * n_e2e / (float(e2e_ms.item()) / 1000.0)

    # ---- config 4: the expert-parallel stack over the same N GPUs ----------
    ep = None
    if not args.no_ep and B == 1:
        del mods, layers
        torch.cuda.empty_cache()
        ep = run_ep(args, rank, world, local, steps=min(K, 5), warmup=3)

    if rank == 0:
        hbm, peak_src = peaks()
        roof = None
        key = next((k2 for k2 in ("tc", "stream", "fused") if k2 in stage_ms), None)
        if key:
            # algorithmic bytes: the k experts' packed weights and scales, the
            # hidden vector in and the output out (intermediates stay on chip
            # or in L2 and are not counted)
            alg = TOPK * EXPERT_BYTES + 2 * H * 2
            ach = alg / (stage_ms[key] / 1000.0) / 1e9
            kernel_names = {"stream": "decode_stream_kernel (one cooperative launch)",
                            "tc": "decode_gateup_tc_kernel + decode_down_tc_kernel (one programmatically "
                                  "dependent pair)",
                            "fused": "moe_decode_fused_kernel"}
            roof = {"bound": "hbm", "kernel": kernel_names[key],
                    "achieved": round(ach, 1), "peak": hbm,
                    "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                    else "of fallback", "unit": "GB/s", "frac": round(ach / hbm, 4),
                    "traffic": NCU_TRAFFIC.get(key), "algorithmic_bytes": alg,
                    "launch_us": round(stage_ms[key] * 1000, 3),
                    "other_paths_us": {k2: round(v * 1000, 3) for k2, v in stage_ms.items() if k2 != key}}
        step_bytes = TOPK * EXPERT_BYTES + 2 * H * 2
        res = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp4(e2m1)+e4m3 scales, fp32 accumulate, bf16 io",
            "data": "synthetic (bf16 N(0,0.02) weights quantized on device; N(0,1) hidden; uniform top-8)",
            "config": decode_config(B, L, world),
            "step_hbm_gbs": round(step_bytes / (ms_max / K / 1000.0) / 1e9, 1),
            "gpu_launches": (2 if tc_path else 1) * K,
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_val, 1), "unit": "tok/s", "steps": n_e2e,
                    "h2d_bytes_per_step": B * H * 2 + B * TOPK * 8 + B * TOPK * 2,
                    "d2h_bytes_per_step": B * H * 2,
                    "path": "Gemma4TextExpertsNVFP4.forward eager, pinned host in/out, sync per step"},
            "roofline": roof,
            "prefill": prefill,
            "decode_batch_sweep": sweep,
            "quantizer": quantizer,
            "ep": ep,
        }
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(args.cpu_seconds, B)
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
