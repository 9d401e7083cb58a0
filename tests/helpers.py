"""Shared test helpers: seeded inputs and torch <-> oracle conversions."""
import numpy as np
import torch

from oracle import numerics as N


def bf16_to_np(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> float32 numpy array of the same values."""
    return t.detach().to(torch.float32).cpu().numpy()


def np_to_bf16(a, device="cuda") -> torch.Tensor:
    bits = N.bf16_bits(np.asarray(a, np.float32)).view(np.int16)
    return torch.from_numpy(bits.copy()).view(torch.bfloat16).to(device)


def bits_to_bf16(bits, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16).copy()).view(torch.bfloat16).to(device)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def randn_bf16(shape, std, seed, device="cuda") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16).to(device)


def max_rel_err(out, ref):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(out - ref)) / max(np.max(np.abs(ref)), 1e-30))


# Output tolerance for GEMM / MoE results against the fp32 dequantize-then-
# matmul oracle: max|err| <= 2e-3 * max|ref|.
TOL = 2e-3


def routing(T, E, k, seed):
    """top-k ids uniform without replacement and softmax(N(0,1)) weights."""
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=g), -1).to(torch.bfloat16)
    return idx, w


def bf16_ulp(x) -> np.ndarray:
    """Spacing of bf16 values at |x| (2^(e-7) for normal x in [2^e, 2^(e+1)))."""
    a = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.exp2(e - 7)


def within_tol_or_ulp(out, ref, tol=TOL) -> bool:
    """max|err| <= tol * max|ref|, where an output one bf16 ulp from the
    reference also passes. An f32 accumulation in another order than the f64
    oracle's sits a few f32 ulps from it and, at a bf16 rounding boundary,
    rounds to the neighbouring bf16 value: one ulp is up to 2^-8 of the value,
    above 2e-3 * max|ref| for outputs near the maximum."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    lim = np.maximum(tol * np.max(np.abs(ref)), bf16_ulp(ref))
    return bool(np.all(np.abs(out - ref) <= lim))


def check_router(probs, w, idx, ref_probs, ref_w, ref_idx, ulps=2, w_tol=1e-2):
    """Router outputs against a reference: probabilities within one bf16 ulp
    of max|ref| ... (``ulps`` ulps); per token the top-k sets agree except
    for experts whose reference probability lies within ``ulps`` bf16 ulps
    of the reference's k-th value (near-ties, where the order of equal
    values or a last-place rounding decides); where the sets agree, the
    weights of each expert agree within ``w_tol`` of the row's max weight.
    Returns the number of tokens whose sets differ."""
    probs, ref_probs = np.asarray(probs, np.float64), np.asarray(ref_probs, np.float64)
    assert np.max(np.abs(probs - ref_probs)) <= ulps * float(bf16_ulp(ref_probs.max()))
    idx, ref_idx = np.asarray(idx), np.asarray(ref_idx)
    w, ref_w = np.asarray(w, np.float64), np.asarray(ref_w, np.float64)
    k = idx.shape[1]
    differ = 0
    for t in range(idx.shape[0]):
        kth = np.sort(ref_probs[t])[::-1][k - 1]
        s, r = set(idx[t].tolist()), set(ref_idx[t].tolist())
        assert len(s) == k
        if s != r:
            differ += 1
            for e in s ^ r:
                assert abs(ref_probs[t, e] - kth) <= ulps * float(bf16_ulp(kth)), (t, e, ref_probs[t, e], kth)
            continue
        a = dict(zip(idx[t].tolist(), w[t].tolist()))
        b = dict(zip(ref_idx[t].tolist(), ref_w[t].tolist()))
        m = max(abs(v) for v in b.values())
        for e in s:
            assert abs(a[e] - b[e]) <= w_tol * m, (t, e, a[e], b[e])
        # descending order of the probabilities behind the weights
        pv = ref_probs[t, idx[t]]
        assert np.all(np.diff(pv) <= ulps * float(bf16_ulp(pv[0])))
    return differ
