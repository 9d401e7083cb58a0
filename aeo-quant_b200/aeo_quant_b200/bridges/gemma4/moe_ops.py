"""Host side of the fused expert forwards: shape checks, workspace, C-ABI calls.

Shared by ``Gemma4TextExpertsNVFP4`` and ``Gemma4TextExpertsFP8``. Each
function restates one reference forward; the arithmetic is in the sm_100a
library.
"""
from __future__ import annotations

import torch

from ... import _capi as A
from ...gpu.quant import quantize_2d_to_nvfp4


_FUSED_WS: dict = {}


def _fused_workspace(lib, device, k, H, I):
    """Zero-initialised workspace of the cooperative decode kernel, one per
    (device, shape). The kernel leaves its counters zero on exit, so the
    buffer is reused by every stream-ordered call (not by overlapping ones)."""
    key = (device.index, k, H, I)
    ws = _FUSED_WS.get(key)
    if ws is None:
        n = lib.aeoq_moe_nvfp4_decode_fused_workspace_size(k, H, I)
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _FUSED_WS[key] = ws
    return ws


_TC_WS: dict = {}
_STREAM_WS: dict = {}

# One-token kernel choice: "tc" (tensor cores, two launches), "stream" (one
# cooperative launch that streams every routed weight into shared memory at
# entry), "fused" (the first cooperative CUDA-core kernel), "chained" (three
# CUDA-core launches); "auto" takes the first that supports the shape, in
# that order (the order of their measured one-token times on a B200).
DECODE_PATH = "auto"


def nvfp4_decode(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, fused=None, path=None):
    """One-token forward (modeling_nvfp4.py:132-186)."""
    A.require_cuda(hidden, top_k_index, top_k_weights, gu, dw)
    lib = A.load()
    if hidden.dtype != torch.bfloat16:
        raise ValueError(f"hidden_states must be bfloat16, got {hidden.dtype}")
    E, two_i, h_half = gu.shape
    H, I = h_half * 2, two_i // 2
    if hidden.shape[-1] != H:
        raise ValueError(f"hidden size {hidden.shape[-1]} != expert hidden size {H}")
    k = top_k_index.shape[-1]
    hidden = hidden.contiguous()
    idx = top_k_index.reshape(-1)[:k].contiguous()
    w = top_k_weights.reshape(-1)[:k].to(torch.bfloat16).contiguous()
    out = torch.empty(1, H, dtype=torch.bfloat16, device=hidden.device)
    path = path or ("fused" if fused else "chained" if fused is False else DECODE_PATH)
    if path in ("auto", "tc") and lib.aeoq_moe_nvfp4_decode_tc_supported(k, H, I):
        key = (hidden.device.index, k, H, I)
        ws = _TC_WS.get(key)
        if ws is None:
            ws = torch.zeros(lib.aeoq_moe_nvfp4_decode_tc_workspace_size(k, H, I), dtype=torch.uint8,
                             device=hidden.device)
            _TC_WS[key] = ws
        A.check(lib.aeoq_moe_nvfp4_decode_tc(
            hidden.data_ptr(), idx.data_ptr(), A.dtype_code(idx.dtype), w.data_ptr(), k,
            gu.data_ptr(), gu_sf.data_ptr(), gu_ts.data_ptr(), A.dtype_code(gu_ts.dtype),
            dw.data_ptr(), dw_sf.data_ptr(), dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype),
            E, H, I, out.data_ptr(), ws.data_ptr(), ws.numel(), A.err_word(hidden.device).data_ptr(),
            A.stream_ptr(hidden.device)))
        return out
    if path == "tc":
        raise ValueError(f"tensor-core decode does not support top_k={k}, hidden={H}, inter={I}")
    if path in ("auto", "stream") and lib.aeoq_moe_nvfp4_decode_stream_supported(k, H, I) and \
            gu_sf.data_ptr() % 16 == 0 and dw_sf.data_ptr() % 16 == 0:
        key = (hidden.device.index, k, H, I)
        ws = _STREAM_WS.get(key)
        if ws is None:
            ws = torch.zeros(lib.aeoq_moe_nvfp4_decode_stream_workspace_size(k, H, I), dtype=torch.uint8,
                             device=hidden.device)
            _STREAM_WS[key] = ws
        A.check(lib.aeoq_moe_nvfp4_decode_stream(
            hidden.data_ptr(), idx.data_ptr(), A.dtype_code(idx.dtype), w.data_ptr(), k,
            gu.data_ptr(), gu_sf.data_ptr(), gu_ts.data_ptr(), A.dtype_code(gu_ts.dtype),
            dw.data_ptr(), dw_sf.data_ptr(), dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype),
            E, H, I, out.data_ptr(), ws.data_ptr(), ws.numel(), A.err_word(hidden.device).data_ptr(),
            A.stream_ptr(hidden.device)))
        return out
    if path == "stream":
        raise ValueError(f"streamed decode does not support top_k={k}, hidden={H}, inter={I}")
    fused = path in ("auto", "fused")
    if fused:
        fused = bool(lib.aeoq_moe_nvfp4_decode_fused_supported(k, H, I))
    if fused:
        ws = _fused_workspace(lib, hidden.device, k, H, I)
        fn, ws_n = lib.aeoq_moe_nvfp4_decode_fused, ws.numel()
    else:
        ws_n = lib.aeoq_moe_nvfp4_decode_workspace_size(k, H, I)
        ws = torch.empty(ws_n, dtype=torch.uint8, device=hidden.device)
        fn = lib.aeoq_moe_nvfp4_decode
    A.check(fn(
        hidden.data_ptr(), idx.data_ptr(), A.dtype_code(idx.dtype), w.data_ptr(), k,
        gu.data_ptr(), gu_sf.data_ptr(), gu_ts.data_ptr(), A.dtype_code(gu_ts.dtype),
        dw.data_ptr(), dw_sf.data_ptr(), dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype),
        E, H, I, out.data_ptr(), ws.data_ptr(), ws_n, A.stream_ptr(hidden.device)))
    return out


class DecodeLauncher:
    """The one-token forward of one expert layer with everything that does
    not change between tokens resolved once: the kernel (the path
    ``nvfp4_decode`` would pick), the weight pointers and dtype codes, the
    workspace and the error word. A call then checks the token's tensors,
    allocates the output and makes one C call: the same launches and bits as
    ``nvfp4_decode``, with less host time per token. Build a new one when
    the weights change (``Gemma4TextExpertsNVFP4`` keys it on the buffers'
    addresses and versions)."""

    def __init__(self, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts):
        A.require_cuda(gu, dw)
        lib = A.load()
        E, two_i, h_half = gu.shape
        self.E, self.H, self.I = E, h_half * 2, two_i // 2
        self.dev = gu.device
        self.lib = lib
        self.k = None
        self.weights = (gu.data_ptr(), gu_sf.data_ptr(), gu_ts.data_ptr(), A.dtype_code(gu_ts.dtype),
                        dw.data_ptr(), dw_sf.data_ptr(), dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype))
        self._keep = (gu, gu_sf, gu_ts, dw, dw_sf, dw_ts)

    def _setup(self, k):
        lib, H, I, dev = self.lib, self.H, self.I, self.dev
        self.fn = None
        if DECODE_PATH in ("auto", "tc") and lib.aeoq_moe_nvfp4_decode_tc_supported(k, H, I):
            self.ws = torch.zeros(lib.aeoq_moe_nvfp4_decode_tc_workspace_size(k, H, I), dtype=torch.uint8,
                                  device=dev)
            self.fn, self.err = lib.aeoq_moe_nvfp4_decode_tc, (A.err_word(dev).data_ptr(),)
        elif DECODE_PATH in ("auto", "stream") and lib.aeoq_moe_nvfp4_decode_stream_supported(k, H, I) and \
                self._keep[1].data_ptr() % 16 == 0 and self._keep[4].data_ptr() % 16 == 0:
            self.ws = torch.zeros(lib.aeoq_moe_nvfp4_decode_stream_workspace_size(k, H, I), dtype=torch.uint8,
                                  device=dev)
            self.fn, self.err = lib.aeoq_moe_nvfp4_decode_stream, (A.err_word(dev).data_ptr(),)
        self.k = k

    def __call__(self, hidden, top_k_index, top_k_weights):
        k = top_k_index.shape[-1]
        if k != self.k:
            self._setup(k)
        if (self.fn is None or hidden.dtype != torch.bfloat16 or hidden.device != self.dev
                or not hidden.is_contiguous() or hidden.shape[-1] != self.H
                or top_k_weights.dtype != torch.bfloat16 or not top_k_index.is_contiguous()
                or not top_k_weights.is_contiguous()):
            gu, gu_sf, gu_ts, dw, dw_sf, dw_ts = self._keep
            return nvfp4_decode(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts)
        out = torch.empty(1, self.H, dtype=torch.bfloat16, device=self.dev)
        A.check(self.fn(hidden.data_ptr(), top_k_index.data_ptr(), A.dtype_code(top_k_index.dtype),
                        top_k_weights.data_ptr(), k, *self.weights, self.E, self.H, self.I, out.data_ptr(),
                        self.ws.data_ptr(), self.ws.numel(), *self.err,
                        torch.cuda.current_stream(self.dev).cuda_stream))
        return out


def pick_tile_n(n_pairs: int, num_experts: int) -> int:
    """Token-tile width of the grouped GEMMs from the mean rows per expert."""
    avg = max(1, n_pairs // max(1, min(num_experts, n_pairs)))
    for bn in (8, 16, 32, 64):
        if avg <= bn:
            return bn
    # the persistent kernel (accumulator double-buffered in TMEM); an MMA
    # costs about the same up to 256 tokens wide, so wide tiles pay once the
    # experts hold more than a 128-row tile on average
    return 128 if avg < 160 else 224


class _Route:
    """Device buffers of one routing: expert-sorted rows of the (token, slot) pairs."""

    def __init__(self, lib, top_k_index, top_k_weights, E, tile_n):
        dev = top_k_index.device
        T, k = top_k_index.shape
        P = T * k
        i32 = dict(dtype=torch.int32, device=dev)
        self.P, self.T, self.k, self.E, self.tile_n = P, T, k, E, tile_n
        self.cnt = torch.empty(E, **i32)
        self.fill = torch.empty(E, **i32)
        self.grp_off = torch.empty(E + 1, **i32)
        self.tile_off = torch.empty(E + 1, **i32)
        self.pair_row = torch.empty(P, **i32)
        self.row_tok = torch.empty(P, **i32)
        self.row_exp = torch.empty(P, **i32)
        self.row_w = torch.empty(P, dtype=torch.bfloat16, device=dev)
        self.ids = top_k_index.contiguous()
        w = top_k_weights.to(torch.bfloat16).contiguous()
        A.check(lib.aeoq_moe_route(self.ids.data_ptr(), A.dtype_code(self.ids.dtype), w.data_ptr(), T, k, E, tile_n,
                                   self.cnt.data_ptr(), self.fill.data_ptr(), self.grp_off.data_ptr(),
                                   self.tile_off.data_ptr(), self.pair_row.data_ptr(), self.row_tok.data_ptr(),
                                   self.row_w.data_ptr(), self.row_exp.data_ptr(), A.stream_ptr(dev)))

    @property
    def n_rows_ptr(self):
        return self.grp_off.data_ptr() + 4 * self.E


def _nvfp4_expert_rows(lib, r, a_packed, a_sf, a_ts, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, one_token_semantics):
    """Grouped expert pipeline over quantized token rows: gather by expert,
    gate_up GEMM with the GeGLU epilogue (per-expert |h| maxima), NVFP4
    re-quantization (per-expert tensor scale, or one shared with
    ``one_token_semantics``), down GEMM weighted by the routing weights.
    Returns the (pairs, H) bf16 outputs in expert-sorted row order
    (``r.pair_row`` maps each (token, slot) pair to its row)."""
    dev = a_packed.device
    E, two_i, h_half = gu.shape
    H, I = h_half * 2, two_i // 2
    P, tile_n = r.P, r.tile_n
    st = A.stream_ptr(dev)
    err = A.err_word(dev)
    gu_atoms = A.weight_atoms(gu_sf, E, 2 * I, H, geglu_inter=I)
    dw_atoms = A.weight_atoms(dw_sf, E, H, I)
    max_tiles = (P + tile_n - 1) // tile_n + E
    a_sorted = torch.empty(P, H // 2, dtype=torch.uint8, device=dev)
    a_sorted_sf = torch.empty(lib.aeoq_nvfp4_act_atoms_size(max_tiles, H, tile_n), dtype=torch.uint8, device=dev)
    A.check(lib.aeoq_gather_rows(a_packed.data_ptr(), a_sf.data_ptr(), r.row_tok.data_ptr(), r.row_exp.data_ptr(),
                                 r.grp_off.data_ptr(), r.tile_off.data_ptr(), tile_n, r.n_rows_ptr, P, H // 2,
                                 H // 16, a_sorted.data_ptr(), a_sorted_sf.data_ptr(), st))
    amax = torch.zeros(E, dtype=torch.int32, device=dev)
    h_sorted = torch.empty(P, I, dtype=torch.bfloat16, device=dev)
    A.check(lib.aeoq_nvfp4_gemm_grouped(a_sorted.data_ptr(), a_sorted_sf.data_ptr(), P, r.grp_off.data_ptr(),
                                        r.tile_off.data_ptr(), tile_n, gu.data_ptr(), gu_atoms.data_ptr(), E, 2 * I, H,
                                        1, a_ts.data_ptr(), A.dtype_code(a_ts.dtype), gu_ts.data_ptr(),
                                        A.dtype_code(gu_ts.dtype), None, None, amax.data_ptr(), h_sorted.data_ptr(),
                                        I * 2, err.data_ptr(), st))
    hq = torch.empty(P, I // 2, dtype=torch.uint8, device=dev)
    hq_sf = torch.empty(lib.aeoq_nvfp4_act_atoms_size(max_tiles, I, tile_n), dtype=torch.uint8, device=dev)
    ts_e = torch.empty(E, dtype=torch.float32, device=dev)
    A.check(lib.aeoq_requant_rows(h_sorted.data_ptr(), I, r.row_exp.data_ptr(), r.grp_off.data_ptr(),
                                  r.tile_off.data_ptr(), tile_n, r.n_rows_ptr, P, amax.data_ptr(), E,
                                  1 if one_token_semantics else 0, hq.data_ptr(), hq_sf.data_ptr(),
                                  ts_e.data_ptr(), st))
    c_sorted = torch.empty(P, H, dtype=torch.bfloat16, device=dev)
    A.check(lib.aeoq_nvfp4_gemm_grouped(hq.data_ptr(), hq_sf.data_ptr(), P, r.grp_off.data_ptr(),
                                        r.tile_off.data_ptr(), tile_n, dw.data_ptr(), dw_atoms.data_ptr(), E, H, I,
                                        2, None, 0, dw_ts.data_ptr(), A.dtype_code(dw_ts.dtype), ts_e.data_ptr(),
                                        r.row_w.data_ptr(), None, c_sorted.data_ptr(), H * 2, err.data_ptr(), st))
    return c_sorted


def nvfp4_experts_grouped(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts,
                          one_token_semantics=False):
    """Expert forward over any number of tokens on the device, no host sync.

    Prefill semantics (modeling_nvfp4.py:188-255): one global activation
    quant, per-expert gate_up, GeGLU, per-expert re-quantized down, weighted
    combine folded in expert order with bf16 rounding after each add. With
    ``one_token_semantics`` the down input shares one tensor scale and the
    combine sums in f32 (modeling_nvfp4.py:132-186).
    """
    A.require_cuda(hidden, top_k_index, top_k_weights, gu, dw)
    lib = A.load()
    dev = hidden.device
    E, two_i, h_half = gu.shape
    H = h_half * 2
    T = hidden.shape[0]
    k = top_k_index.shape[-1]
    r = _Route(lib, top_k_index.reshape(T, k), top_k_weights.reshape(T, k), E, pick_tile_n(T * k, E))
    hp, hs, hts = quantize_2d_to_nvfp4(hidden)                                   # (:203-206)
    c_sorted = _nvfp4_expert_rows(lib, r, hp, hs, hts, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, one_token_semantics)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    A.check(lib.aeoq_moe_combine(c_sorted.data_ptr(), r.pair_row.data_ptr(), r.ids.data_ptr(),
                                 A.dtype_code(r.ids.dtype), T, k, H, 1 if one_token_semantics else 0,
                                 out.data_ptr(), A.stream_ptr(dev)))
    return out


def nvfp4_prefill(hidden, top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts, num_experts):
    """Many-token forward (modeling_nvfp4.py:188-255), all on the device."""
    if hidden.dtype != torch.bfloat16:
        raise ValueError(f"hidden_states must be bfloat16, got {hidden.dtype}")
    if gu.shape[0] != num_experts:
        raise ValueError(f"gate_up_proj holds {gu.shape[0]} experts, config says {num_experts}")
    return nvfp4_experts_grouped(hidden.contiguous(), top_k_index, top_k_weights, gu, gu_sf, gu_ts, dw, dw_sf,
                                 dw_ts)


# ---------------------------------------------------------------- FP8 experts
def fp8_scale_rows(scale: torch.Tensor, E: int, N: int) -> torch.Tensor:
    """Per-output-channel weight scales as a flat f32 (E * N) tensor: accepts
    the checkpoint's (E, N, 1) bf16 buffer or the preconverted (E, 1, N) f32
    one (loader.py:47-64); the values are the same."""
    if scale.numel() != E * N:
        raise ValueError(f"expected {E * N} weight scales, got shape {tuple(scale.shape)}")
    return scale.reshape(E * N).to(torch.float32).contiguous()


def fp8_linear(x_bf16: torch.Tensor, w_fp8: torch.Tensor, scale_w: torch.Tensor) -> torch.Tensor:
    """``_fp8_linear`` (modeling.py:89-108): per-row dynamic e4m3 input
    quantization, then bf16((acc * sa[m]) * sb[n]) on the tensor cores."""
    A.require_cuda(x_bf16, w_fp8, scale_w)
    lib = A.load()
    if x_bf16.dtype != torch.bfloat16:
        raise ValueError(f"_fp8_linear expects bfloat16 input, got {x_bf16.dtype}")
    if w_fp8.dim() != 2:
        raise ValueError(f"w_fp8 must be 2D (N, K), got shape {tuple(w_fp8.shape)}")
    N, K = w_fp8.shape
    x2 = x_bf16.reshape(-1, x_bf16.shape[-1]).contiguous()
    M = x2.shape[0]
    if x2.shape[1] != K:
        raise ValueError(f"input features {x2.shape[1]} != weight in_features {K}")
    dev = x2.device
    st = A.stream_ptr(dev)
    sb = scale_w.reshape(N).to(torch.float32).contiguous()
    q = torch.empty(M, K, dtype=torch.uint8, device=dev)
    sa = torch.empty(M, dtype=torch.float32, device=dev)
    A.check(lib.aeoq_fp8_quantize_rows_gather(x2.data_ptr(), K, None, None, M, K, q.data_ptr(), K, sa.data_ptr(), st))
    out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    wv = w_fp8.contiguous().view(torch.uint8)
    A.check(lib.aeoq_fp8_gemm(q.data_ptr(), sa.data_ptr(), M, wv.data_ptr(), sb.data_ptr(), N, K, out.data_ptr(),
                              A.err_word(dev).data_ptr(), st))
    return out.reshape(*x_bf16.shape[:-1], N)


def fp8_experts_grouped(hidden, top_k_index, top_k_weights, gu, gu_sb, dw, dw_sb):
    """``Gemma4TextExpertsFP8.forward`` (modeling.py:110-146) on the device,
    no host sync: route by expert, per-row e4m3 quantization of the gathered
    tokens, grouped gate_up GEMM with the GeGLU epilogue, per-row
    re-quantization, grouped down GEMM weighted by the routing weights, and
    the bf16 ``index_add_`` fold in ascending expert order.

    ``gu`` (E, 2I, H) and ``dw`` (E, H, I) e4m3 (any 1-byte view);
    ``gu_sb`` / ``dw_sb`` flat f32 (E * 2I) / (E * H)."""
    A.require_cuda(hidden, top_k_index, top_k_weights, gu, dw)
    lib = A.load()
    dev = hidden.device
    E, two_i, H = gu.shape
    I = two_i // 2
    T = hidden.shape[0]
    k = top_k_index.shape[-1]
    P = T * k
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if T == 0:
        return out
    st = A.stream_ptr(dev)
    err = A.err_word(dev)
    tile_n = pick_tile_n(P, E)
    r = _Route(lib, top_k_index.reshape(T, k), top_k_weights.reshape(T, k), E, tile_n)
    hidden = hidden.contiguous()
    gu8 = gu.detach().contiguous().view(torch.uint8)
    dw8 = dw.detach().contiguous().view(torch.uint8)
    xq = torch.empty(P, H, dtype=torch.uint8, device=dev)
    sa = torch.empty(P, dtype=torch.float32, device=dev)
    A.check(lib.aeoq_fp8_quantize_rows_gather(hidden.data_ptr(), H, r.row_tok.data_ptr(), r.n_rows_ptr, P, H,
                                              xq.data_ptr(), H, sa.data_ptr(), st))           # (:101-104)
    h = torch.empty(P, I, dtype=torch.bfloat16, device=dev)
    A.check(lib.aeoq_fp8_gemm_grouped(xq.data_ptr(), sa.data_ptr(), P, r.grp_off.data_ptr(), r.tile_off.data_ptr(),
                                      tile_n, gu8.data_ptr(), gu_sb.data_ptr(), E, 2 * I, H, 1, None, h.data_ptr(),
                                      I * 2, err.data_ptr(), st))                           # (:124-131)
    hq = torch.empty(P, I, dtype=torch.uint8, device=dev)
    sh = torch.empty(P, dtype=torch.float32, device=dev)
    A.check(lib.aeoq_fp8_quantize_rows_gather(h.data_ptr(), I, None, r.n_rows_ptr, P, I, hq.data_ptr(), I,
                                              sh.data_ptr(), st))
    c = torch.empty(P, H, dtype=torch.bfloat16, device=dev)
    A.check(lib.aeoq_fp8_gemm_grouped(hq.data_ptr(), sh.data_ptr(), P, r.grp_off.data_ptr(), r.tile_off.data_ptr(),
                                      tile_n, dw8.data_ptr(), dw_sb.data_ptr(), E, H, I, 2, r.row_w.data_ptr(),
                                      c.data_ptr(), H * 2, err.data_ptr(), st))              # (:133-140)
    A.check(lib.aeoq_moe_combine(c.data_ptr(), r.pair_row.data_ptr(), r.ids.data_ptr(), A.dtype_code(r.ids.dtype),
                                 T, k, H, 0, out.data_ptr(), st))                          # (:142-145)
    return out
