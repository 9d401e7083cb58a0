"""CPU restatement of the Gemma-4 router (numpy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The router is not aeo_quant code: it is HF transformers 5.5.0
``Gemma4TextRouter.forward`` (``models/gemma4/modeling_gemma4.py:1296-1316``)
with ``Gemma4RMSNorm`` (:166-175, ``with_scale=False``), the caller that
produces ``top_k_index`` / ``top_k_weights`` for the expert modules
(:1379-1383). Every bf16 rounding point of the eager ops is kept; sums are
evaluated in float64 and rounded once, so the oracle sits within the
ordering error of any float32 implementation.

Arrays: x (T, H) float32 holding bf16 values; scale (H,), proj_w (E, H),
per_expert_scale (E,) float32 holding bf16 values.
"""
from __future__ import annotations

import numpy as np

from .numerics import F32, bf16


def gemma4_router(x, scale, proj_w, per_expert_scale, top_k: int, eps: float = 1e-6):
    """Returns (probs (T,E), top_k_weights (T,k), top_k_index (T,k) int64).
    Equal probabilities are ordered by the lower expert id."""
    x = np.asarray(x, F32)
    T, H = x.shape
    ms = F32((x.astype(np.float64) ** 2).sum(-1) / H) + F32(eps)            # :167
    r = (1.0 / np.sqrt(ms.astype(np.float64))).astype(F32)                   # :169
    n = bf16(x * r[:, None])                                                 # :172-175
    y = bf16(bf16(n * np.asarray(scale, F32)[None, :]) * F32(H ** -0.5))     # :1299-1300
    logits = bf16((y.astype(np.float64) @ np.asarray(proj_w, np.float64).T).astype(F32))   # :1302
    z = logits.astype(np.float64) - logits.max(-1, keepdims=True)
    e = np.exp(z)
    probs = bf16((e / e.sum(-1, keepdims=True)).astype(F32))                 # :1303
    E = probs.shape[1]
    order = np.lexsort((np.broadcast_to(np.arange(E), probs.shape), -probs), axis=-1)
    idx = order[:, :top_k].astype(np.int64)                                  # :1306-1310
    val = np.take_along_axis(probs, idx, -1)
    den = bf16(val.astype(np.float64).sum(-1, keepdims=True).astype(F32))    # :1313
    w = bf16(val / den)
    w = bf16(w * np.asarray(per_expert_scale, F32)[idx])                     # :1316
    return probs, w, idx
