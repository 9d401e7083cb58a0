"""Gemma-4 router on one fused kernel.

``Gemma4TextRouterB200`` is HF transformers' ``Gemma4TextRouter`` (5.5.0,
``models/gemma4/modeling_gemma4.py:1283-1316``) with the same parameters
(``proj.weight``, ``scale``, ``per_expert_scale``) and the same outputs
``(router_probabilities, top_k_weights, top_k_index)``. Its forward is
``aeoq_gemma4_router``: RMS norm, scale, projection, softmax, top-k,
renormalisation and per-expert scale in one launch, in place of about ten
eager launches. The router sits in front of the swapped expert modules in
every ``Gemma4TextDecoderLayer`` (:1379-1383); ``loader.swap_routers``
installs it on a built model and ``loader.gemma4_router_class_swap`` during
``from_pretrained``.
"""
from __future__ import annotations

import torch
from transformers.models.gemma4.modeling_gemma4 import Gemma4TextRouter

from ... import _capi as A


def router_supported(router) -> bool:
    """True if the fused kernel takes this router: bfloat16 parameters
    (``proj.weight``, ``scale``, ``per_expert_scale``), hidden size H a
    multiple of 8 with 2E + 128 <= H <= 6144, E a multiple of 8 up to 256,
    top_k <= min(E, 32) (the limits ``aeoq_gemma4_router`` checks). A router
    loaded in another dtype keeps HF's forward."""
    E, H = router.proj.weight.shape
    k = int(router.config.top_k_experts)
    if any(t.dtype != torch.bfloat16 for t in (router.proj.weight, router.scale, router.per_expert_scale)):
        return False
    return (H % 8 == 0 and 2 * E + 128 <= H <= 6144 and E % 8 == 0 and E <= 256 and 1 <= k <= min(E, 32))


# Above this many tokens HF's eager forward is faster: its 2816 -> 128
# projection is a cuBLAS GEMM, while the fused kernel runs it on CUDA cores.
# Measured on a B200 (``bench.py --workload router``, CUDA-graph replays):
# fused 38.6 us vs HF 61.9 us at 512 tokens, 148 us vs 102 us at 2048; the
# two cross near 1000 tokens.
FUSED_MAX_TOKENS = 768


class Gemma4TextRouterB200(Gemma4TextRouter):
    """Gemma4TextRouter with a fused CUDA forward (bf16 only) for up to
    ``FUSED_MAX_TOKENS`` tokens; larger batches (prefill) take HF's eager
    forward, which is faster there."""

    def forward(self, hidden_states: torch.Tensor):
        x = hidden_states
        if x.dim() == 2 and x.shape[0] > FUSED_MAX_TOKENS:
            return Gemma4TextRouter.forward(self, x)
        if x.dim() != 2:
            raise ValueError(f"router expects (tokens, hidden), got shape {tuple(x.shape)}")
        w = self.proj.weight
        for name, t in (("hidden_states", x), ("proj.weight", w), ("scale", self.scale),
                        ("per_expert_scale", self.per_expert_scale)):
            if t.dtype != torch.bfloat16:
                raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
            if not t.is_cuda:
                raise ValueError(f"{name} must be a CUDA tensor")
        if x.stride(-1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
            x = x.contiguous() if x.stride(-1) != 1 else x.clone()
        T, H = x.shape
        E = w.shape[0]
        k = self.config.top_k_experts
        dev = x.device
        probs = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
        top_w = torch.empty(T, k, dtype=torch.bfloat16, device=dev)
        top_i = torch.empty(T, k, dtype=torch.int64, device=dev)
        lib = A.load()
        A.check(lib.aeoq_gemma4_router(x.data_ptr(), x.stride(0), self.scale.contiguous().data_ptr(),
                                       w.contiguous().data_ptr(), self.per_expert_scale.contiguous().data_ptr(),
                                       T, H, E, k, float(self.eps), float(self.scalar_root_size),
                                       probs.data_ptr(), top_w.data_ptr(), top_i.data_ptr(), A.stream_ptr(dev)))
        return probs, top_w, top_i
