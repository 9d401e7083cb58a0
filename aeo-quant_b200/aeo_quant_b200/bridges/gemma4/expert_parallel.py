"""Expert-parallel NVFP4 expert layer: experts sharded over the ranks of a
process group, tokens sharded by sequence, NCCL all-to-all dispatch and
combine.

Semantics are those of the one-GPU prefill forward
(aeo_quant ``src/aeo_quant/bridges/gemma4/modeling_nvfp4.py:188-255``) over
the union of all ranks' tokens:

* the activation tensor scale comes from the global amax (one
  all-reduce(max) of a scalar; ``quantize_2d_to_nvfp4`` over the whole
  batch, :203-206), and each rank quantizes its own tokens with it;
* each token is sent once to every rank that owns at least one of its
  experts, NVFP4-packed (H/2 bytes of E2M1 plus H/16 e4m3 scales, 3.6x
  fewer bytes than bf16), with the local ids and routing weights of its
  experts there; an expert's rows therefore all meet on one rank, so its
  per-expert down re-quantization (:239-244) sees exactly the rows it would
  on one GPU, and every expert output is bit for bit the one-GPU value;
* the owning rank folds the weighted outputs of a token's experts it holds
  (ascending expert id, bf16 rounding after each add, as ``index_add_``
  does, :250-253) and sends back ONE row per (token, rank); the home rank
  folds those partial rows in rank order with the same rounding.

Only the association of the final fold differs from one GPU: the result
is within the bf16 rounding of up to k adds of the one-GPU forward (a few
ulps), and the bytes on the wire are one row per (token, owning rank) each
way instead of one per (token, expert).

By default rank r owns experts [r * E/world, (r+1) * E/world). A placement
(``owner[e]`` = the rank holding expert e, E/world experts per rank, e.g.
from ``balanced_placement`` for skewed routing) may replace that; a rank
then holds its experts in ascending id order. Pairs whose expert id is
outside [0, E) are dropped (:209-211). ``ep_moe_forward`` is the
orchestration shared by every backend; the expert arithmetic, the payload
codec and the folds are supplied by an ``ops`` object (``NVFP4EpOps`` for
the CUDA library).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ... import _capi as A
from ...gpu.quant import _nvfp4_quantize_rows
from . import moe_ops


def _all_to_all_rows(rows: torch.Tensor, send_counts, recv_counts, group) -> torch.Tensor:
    out = torch.empty((sum(recv_counts),) + tuple(rows.shape[1:]), dtype=rows.dtype, device=rows.device)
    dist.all_to_all_single(out, rows.contiguous(), list(recv_counts), list(send_counts), group=group)
    return out


def contiguous_placement(num_experts: int, world: int) -> torch.Tensor:
    """owner[e] = e // (E/world): rank r holds experts [r*E/world, (r+1)*E/world)."""
    if num_experts % world:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    return torch.arange(num_experts) // (num_experts // world)


def balanced_placement(load, world: int) -> torch.Tensor:
    """A placement with E/world experts per rank that evens out the ranks'
    expected rows: experts by descending ``load`` (ties by id) each go to
    the least-loaded rank that still has room (ties by rank). ``load`` is
    any per-expert weight, e.g. a routing histogram. Returns owner (E,)
    int64 on the host."""
    load = torch.as_tensor(load, dtype=torch.float64).reshape(-1).cpu()
    E = load.numel()
    if E % world:
        raise ValueError(f"num_experts ({E}) must be divisible by the world size ({world})")
    cap = E // world
    order = sorted(range(E), key=lambda e: (-float(load[e]), e))
    owner = torch.empty(E, dtype=torch.int64)
    tot = [0.0] * world
    room = [cap] * world
    for e in order:
        r = min((r for r in range(world) if room[r]), key=lambda r: (tot[r], r))
        owner[e] = r
        tot[r] += float(load[e])
        room[r] -= 1
    return owner


def local_index(owner: torch.Tensor, world: int) -> torch.Tensor:
    """local[e] = position of expert e among its owner's experts (ascending
    id). Raises ValueError unless every rank owns E/world experts."""
    owner = torch.as_tensor(owner, dtype=torch.int64).reshape(-1).cpu()
    E = owner.numel()
    if E % world or bool(((owner < 0) | (owner >= world)).any()):
        raise ValueError("placement must map every expert to a rank in [0, world)")
    counts = torch.bincount(owner, minlength=world)
    if bool((counts != E // world).any()):
        raise ValueError(f"placement must give every rank {E // world} experts, got {counts.tolist()}")
    local = torch.empty(E, dtype=torch.int64)
    seen = [0] * world
    for e in range(E):
        r = int(owner[e])
        local[e] = seen[r]
        seen[r] += 1
    return local


def plan_dispatch(top_k_index: torch.Tensor, num_experts: int, world: int, owner: torch.Tensor | None = None):
    """Send order of the (token, slot) pairs, grouped by owning rank
    (``owner`` (E,) as from ``balanced_placement``; contiguous blocks when
    None).

    Returns ``(send_pairs, send_counts, dest)``: pair indices (t * k + j) in
    send order (by destination rank, then pair index), pairs per destination
    rank, and each pair's destination (``world`` for dropped pairs)."""
    if num_experts % world:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    e_loc = num_experts // world
    ids = top_k_index.reshape(-1).to(torch.int64)
    n = ids.numel()
    valid = (ids >= 0) & (ids < num_experts)
    if owner is None:
        dest = torch.where(valid, torch.div(ids, e_loc, rounding_mode="floor"), torch.full_like(ids, world))
    else:
        owner = owner.to(ids.device)
        dest = torch.where(valid, owner[ids.clamp(0, num_experts - 1)], torch.full_like(ids, world))
    key = dest * n + torch.arange(n, device=ids.device)
    order = torch.argsort(key)
    counts = torch.bincount(dest, minlength=world + 1)[:world]
    n_send = int(counts.sum().item())
    return order[:n_send], counts, dest


def global_amax(hidden: torch.Tensor, group) -> torch.Tensor:
    """max |hidden| over every rank's tokens as a 1-element f32 tensor (one
    all-reduce(max)). A rank without tokens (decode with fewer tokens than
    ranks) contributes 0 and still joins the collective, so no peer waits."""
    if hidden.numel():
        amax = hidden.abs().amax().to(torch.float32).reshape(1)
    else:
        amax = torch.zeros(1, dtype=torch.float32, device=hidden.device)
    dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=group)
    return amax


def plan_token_dispatch(top_k_index: torch.Tensor, num_experts: int, world: int, owner: torch.Tensor | None = None):
    """Send list of one expert-parallel layer: every (token, rank) where the
    rank owns at least one of the token's experts, ordered by rank, then
    token.

    Returns ``(send_tok, send_dest, counts, local_ids)``: the token and the
    destination of each send, sends per destination rank, and per send the k
    local expert ids on the destination (``E/world``, an id the grouped
    forward drops, where the slot's expert lives elsewhere or is invalid)."""
    if num_experts % world:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    e_loc = num_experts // world
    ids = top_k_index.to(torch.int64)
    T, k = ids.shape
    dev = ids.device
    valid = (ids >= 0) & (ids < num_experts)
    safe = ids.clamp(0, num_experts - 1)
    if owner is None:
        dest = torch.div(safe, e_loc, rounding_mode="floor")
        local = safe - dest * e_loc
    else:
        owner = torch.as_tensor(owner, dtype=torch.int64).reshape(-1)
        dest = owner.to(dev)[safe]
        local = local_index(owner, world).to(dev)[safe]
    dest = torch.where(valid, dest, torch.full_like(dest, world))
    present = torch.zeros(world + 1, T, dtype=torch.bool, device=dev)
    present[dest, torch.arange(T, device=dev).unsqueeze(1).expand(T, k)] = True
    sel = torch.nonzero(present[:world].reshape(-1)).reshape(-1)    # rank-major, then token
    send_tok = sel % T
    send_dest = torch.div(sel, T, rounding_mode="floor")
    counts = torch.bincount(send_dest, minlength=world)
    lid = torch.where(dest[send_tok] == send_dest.unsqueeze(1), local[send_tok], torch.full_like(local[send_tok], e_loc))
    return send_tok, send_dest, counts, lid.to(torch.int32)


def plan_dense_dispatch(top_k_index: torch.Tensor, num_experts: int, world: int, owner: torch.Tensor | None = None):
    """Fixed-layout send plan for ranks that all hold the same number of
    tokens T: row r * T + t of the send buffer carries token t to rank r
    whether or not r owns one of its experts, so no split size depends on
    the routing and nothing is read back to the host.

    Returns ``(local_ids, present)``: (world, T, k) local expert ids on each
    rank (``E/world``, dropped by the grouped forward, where the slot's
    expert lives elsewhere or is invalid) and (world, T) whether rank r owns
    any of token t's experts."""
    if num_experts % world:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by the world size ({world})")
    e_loc = num_experts // world
    ids = top_k_index.to(torch.int64)
    dev = ids.device
    valid = (ids >= 0) & (ids < num_experts)
    safe = ids.clamp(0, num_experts - 1)
    if owner is None:
        dest = torch.div(safe, e_loc, rounding_mode="floor")
        local = safe - dest * e_loc
    else:
        owner = torch.as_tensor(owner, dtype=torch.int64).reshape(-1)
        dest = owner.to(dev)[safe]
        local = local_index(owner, world).to(dev)[safe]
    dest = torch.where(valid, dest, torch.full_like(dest, world))
    on = dest.unsqueeze(0) == torch.arange(world, device=dev).view(world, 1, 1)       # (world, T, k)
    lid = torch.where(on, local.unsqueeze(0), torch.full_like(local, e_loc).unsqueeze(0))
    return lid.to(torch.int32), on.any(-1)


def _ep_dense(hidden, top_k_index, top_k_weights, num_experts, group, ops, owner, my_experts, mark):
    """``ep_moe_forward`` for equal token counts on every rank: fixed-size
    all-to-alls, no host synchronisation (see ``plan_dense_dispatch``)."""
    world = dist.get_world_size(group)
    T, k = top_k_index.shape
    dev = hidden.device
    lid, present = plan_dense_dispatch(top_k_index, num_experts, world, owner)
    ts = ops.tensor_scale(global_amax(hidden, group), hidden.dtype)
    wbits = top_k_weights.to(torch.bfloat16).contiguous().view(torch.int16).to(torch.int32)
    meta = torch.cat([lid.reshape(world * T, k), wbits.unsqueeze(0).expand(world, T, k).reshape(world * T, k)], 1)
    # every rank receives every rank's quantized rows (block r = rank r's
    # tokens): an all-gather, with no per-destination copy of the payload
    recv_payload = []
    for p in ops.encode(hidden, ts):
        p = p.contiguous()
        r = torch.empty((world * T, *p.shape[1:]), dtype=p.dtype, device=dev)
        dist.all_gather_into_tensor(r, p, group=group)
        recv_payload.append(r)
    recv_meta = torch.empty_like(meta)
    dist.all_to_all_single(recv_meta, meta, group=group)
    recv_lid = recv_meta[:, :k].contiguous()
    recv_w = recv_meta[:, k:].to(torch.int16).view(torch.bfloat16).contiguous()
    mark("experts")
    partial = ops.experts(recv_payload, recv_lid, recv_w, ts, my_experts, pairs_hint=T * k)   # (world * T, H)

    mark("combine")
    back = torch.empty_like(partial)
    dist.all_to_all_single(back, partial, group=group)   # block r: my tokens as rank r folded them
    rows = (torch.arange(world, device=dev).view(world, 1) * T + torch.arange(T, device=dev).view(1, T))
    slot_row = torch.where(present, rows, torch.full_like(rows, -1)).T.to(torch.int32).contiguous()
    out = ops.fold(back, slot_row, T, world)
    mark("end")
    return out


def ep_moe_forward(hidden, top_k_index, top_k_weights, *, num_experts: int, group, ops, owner=None, mark=None,
                   equal_tokens: bool = False):
    """One expert-parallel MoE layer over ``group`` (see module docstring).
    ``owner``: optional placement (E,) of experts on ranks. ``mark``: optional
    callable taking a phase name ("dispatch", "experts", "combine", "end"),
    called where each phase starts (a profiler hook, e.g. recording CUDA
    events). ``equal_tokens``: every rank passes the same number of tokens
    (sequence-sharded prefill); the layer then uses fixed-size all-to-alls
    and never synchronises with the host. Otherwise each layer reads the
    split sizes back once."""
    if mark is None:
        def mark(_):
            return None
    mark("dispatch")
    if equal_tokens:
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if owner is None:
            e_loc = num_experts // world
            my_experts = torch.arange(rank * e_loc, (rank + 1) * e_loc)
        else:
            owner = torch.as_tensor(owner, dtype=torch.int64).reshape(-1).cpu()
            my_experts = torch.nonzero(owner == rank).reshape(-1)
        return _ep_dense(hidden, top_k_index, top_k_weights, num_experts, group, ops, owner, my_experts, mark)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    e_loc = num_experts // world
    T, k = top_k_index.shape
    dev = hidden.device
    if owner is None:
        my_experts = torch.arange(rank * e_loc, (rank + 1) * e_loc)
    else:
        owner = torch.as_tensor(owner, dtype=torch.int64).reshape(-1).cpu()
        my_experts = torch.nonzero(owner == rank).reshape(-1)
    send_tok, send_dest, send_counts, lid = plan_token_dispatch(top_k_index, num_experts, world, owner)

    # counts: one small all-to-all; everything that does not need the split
    # sizes on the host (the global scale, the quantized rows in send order,
    # the metadata) is queued before the one host read of both split lists,
    # so the device stays busy while the host waits
    recv_counts_t = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts_t, send_counts, group=group)
    ts = ops.tensor_scale(global_amax(hidden, group), hidden.dtype)
    send_payload = [p[send_tok] for p in ops.encode(hidden, ts)]   # per-token rows, in send order
    wbits = top_k_weights.to(torch.bfloat16).contiguous().view(torch.int16).to(torch.int32)
    meta = torch.cat([lid, wbits[send_tok]], dim=1)      # (n_send, 2k) int32
    both = torch.cat([send_counts, recv_counts_t]).tolist()
    sc, rc = both[:world], both[world:]

    recv_payload = [_all_to_all_rows(p, sc, rc, group) for p in send_payload]
    recv_meta = _all_to_all_rows(meta, sc, rc, group)
    recv_lid = recv_meta[:, :k].contiguous()
    recv_w = recv_meta[:, k:].to(torch.int16).view(torch.bfloat16).contiguous()
    mark("experts")
    partial = ops.experts(recv_payload, recv_lid, recv_w, ts, my_experts, pairs_hint=T * k)   # (n_recv, H)

    mark("combine")
    back = _all_to_all_rows(partial, rc, sc, group)      # in this rank's send order
    slot_row = torch.full((T, world), -1, dtype=torch.int32, device=dev)
    slot_row[send_tok, send_dest] = torch.arange(send_tok.numel(), dtype=torch.int32, device=dev)
    out = ops.fold(back, slot_row, T, world)
    mark("end")
    return out


class NVFP4EpOps:
    """The CUDA library's arithmetic for ``ep_moe_forward``: the rank's
    local experts (E/world of them) with the reference's buffers."""

    def __init__(self, gu, gu_sf, gu_ts, dw, dw_sf, dw_ts):
        self.gu, self.gu_sf, self.gu_ts = gu, gu_sf, gu_ts
        self.dw, self.dw_sf, self.dw_ts = dw, dw_sf, dw_ts
        self.lib = A.load()

    def tensor_scale(self, amax, dtype):
        # ts = amax / 2688 in the input dtype, at least 1e-12 (quant.py:167-168)
        return (amax[0].to(dtype) / 2688.0).clamp(min=1e-12)

    def encode(self, hidden, ts):
        packed, sf, _ = _nvfp4_quantize_rows(hidden.contiguous(), ts)
        return [packed, sf.view(torch.uint8)]

    def experts(self, payload, local_ids, weights, ts, my_experts, pairs_hint=None):
        """Grouped forward of the received tokens over this rank's experts,
        then each token's weighted outputs folded (ascending expert id, bf16
        after each add). ``pairs_hint``: the expected number of valid
        (token, expert) pairs, which picks the token-tile width (any width
        gives the same bits)."""
        packed, sf = payload
        n, k = local_ids.shape
        H = self.dw.shape[1]
        dev = packed.device
        out = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        if n == 0:
            return out
        E = self.gu.shape[0]
        hint = pairs_hint if pairs_hint is not None else n * k // 2
        r = moe_ops._Route(self.lib, local_ids, weights, E, moe_ops.pick_tile_n(max(1, hint), E))
        c_sorted = moe_ops._nvfp4_expert_rows(self.lib, r, packed, sf, ts, self.gu, self.gu_sf, self.gu_ts,
                                              self.dw, self.dw_sf, self.dw_ts, False)
        A.check(self.lib.aeoq_moe_combine(c_sorted.data_ptr(), r.pair_row.data_ptr(), r.ids.data_ptr(),
                                          A.dtype_code(r.ids.dtype), n, k, H, 0, out.data_ptr(), A.stream_ptr(dev)))
        return out

    def fold(self, rows, slot_row, T, world):
        """out[t] = the partial rows of token t's ranks folded in rank order
        (bf16 after each add)."""
        H = self.dw.shape[1]
        dev = slot_row.device
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        if T == 0:
            return out
        if rows.shape[0] == 0:
            rows = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
        ranks = torch.arange(world, dtype=torch.int32, device=dev).expand(T, world).contiguous()
        A.check(self.lib.aeoq_moe_combine(rows.contiguous().data_ptr(), slot_row.contiguous().data_ptr(),
                                          ranks.data_ptr(), A.I32, T, world, H, 0, out.data_ptr(),
                                          A.stream_ptr(dev)))
        return out


class ExpertParallelNVFP4(torch.nn.Module):
    """One rank's share of an expert-parallel ``Gemma4TextExpertsNVFP4``.

    Holds experts [rank * E/world, (rank+1) * E/world), or with ``owner``
    the experts e with owner[e] == rank in ascending id order, with the
    reference's buffer names (first dimension E/world); ``forward`` takes
    this rank's tokens and returns their outputs. With ``equal_tokens`` every
    rank must pass the same number of tokens, and the layer runs without a
    host synchronisation (fixed-size all-to-alls)."""

    def __init__(self, local_experts, num_experts: int, group=None, owner=None, equal_tokens: bool = False):
        super().__init__()
        self.local = local_experts
        self.num_experts = num_experts
        self.group = group
        self.owner = None if owner is None else torch.as_tensor(owner, dtype=torch.int64).reshape(-1).cpu()
        self.mark = None   # optional phase hook passed to ep_moe_forward
        self.equal_tokens = equal_tokens

    def forward(self, hidden_states, top_k_index, top_k_weights):
        m = self.local
        if hidden_states.dtype != torch.bfloat16:
            raise ValueError(f"hidden_states must be bfloat16, got {hidden_states.dtype}")
        ops = NVFP4EpOps(m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2,
                         m.down_proj, m.down_proj_scale, m.down_proj_scale_2)
        return ep_moe_forward(hidden_states, top_k_index, top_k_weights, num_experts=self.num_experts,
                              group=self.group, ops=ops, owner=self.owner, mark=self.mark,
                              equal_tokens=self.equal_tokens)
