"""One rank of the CPU (gloo) expert-parallel test: runs the shared
orchestration ``ep_moe_forward`` with oracle arithmetic on this rank's
tokens and saves its output rows. Launched by test_expert_parallel.py as
``python ep_worker.py RANK WORLD PORT OUT.npz CASE``."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, ROOT, os.path.join(ROOT, "aeo-quant_b200")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import moe as OM  # noqa: E402
from oracle import numerics as N  # noqa: E402
from oracle import quant as OQ  # noqa: E402
from oracle.gemm import nvfp4_gemm, nvfp4_linear  # noqa: E402


def case_inputs(case):
    """Deterministic layer and tokens shared by the workers and the test.
    Case 2 is case 1's skewed routing, run with a balanced placement. Case 3
    has a single token, so with two ranks one of them holds none."""
    if case == 2:
        return case_inputs(1)
    g = np.load(os.path.join(HERE, "golden", "moe_golden.npz"))
    m = OM.NVFP4Experts(g["nv/gate_up_proj"], g["nv/gate_up_proj_scale"], g["nv/gate_up_proj_scale_2"][0],
                        g["nv/down_proj"], g["nv/down_proj_scale"], g["nv/down_proj_scale_2"][0])
    E, H = m.num_experts, m.down_proj.shape[1]
    rng = np.random.default_rng(7 + case)
    T, k = (1 if case == 3 else 12), 4
    hidden = N.bf16(rng.standard_normal((T, H)).astype(np.float32))
    if case in (0, 3):      # uniform routing
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    else:              # skewed: most pairs on rank 0's experts, one dropped id (== E)
        ids = np.stack([np.r_[rng.permutation(3)[:k - 1], 3 + (t % 5)] for t in range(T)])
        ids[2, 1] = E
    w = N.bf16(rng.dirichlet(np.ones(k), size=T).astype(np.float32))
    return m, hidden, ids, w


def pair_outputs(m, hidden, ids, wts, ts=None):
    """Weighted down output of every valid (token, slot) pair, the one-GPU
    prefill's per-expert steps (modeling_nvfp4.py:203-249): {(t, j): row}."""
    hp, hs, hts = OQ.quantize_nvfp4(hidden, "bf16", ts=ts)
    out = {}
    for e in np.unique(ids):
        if e < 0 or e >= m.num_experts:
            continue
        pos, tok = np.nonzero(ids.T == e)
        gu = nvfp4_gemm(hp[tok], hs[tok], hts, m.gate_up_proj[e], m.gate_up_proj_scale[e], m.gate_up_proj_scale_2)
        d = nvfp4_linear(OM.geglu(gu), m.down_proj[e], m.down_proj_scale[e], m.down_proj_scale_2)
        d = N.bf16(d * wts[tok, pos][:, None])
        for i, (t, j) in enumerate(zip(tok, pos)):
            out[(int(t), int(j))] = d[i]
    return out


def ep_order_reference(m, hidden, ids, wts, owner, world):
    """The expert-parallel result restated on one process: per token, each
    owning rank folds its experts' rows (ascending id, bf16 after each add),
    then the partials are folded in rank order."""
    pairs = pair_outputs(m, hidden, ids, wts)
    T, H = hidden.shape[0], m.down_proj.shape[1]
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for r in range(world):
            slots = sorted((int(ids[t, j]), j) for j in range(ids.shape[1])
                           if 0 <= ids[t, j] < m.num_experts and int(owner[ids[t, j]]) == r)
            if not slots:
                continue
            part = np.zeros(H, np.float32)
            for _, j in slots:
                part = N.bf16(part + pairs[(t, j)])
            acc = N.bf16(acc + part)
        out[t] = acc
    return out


class OracleEpOps:
    """Oracle arithmetic for ep_moe_forward (the rank's experts only)."""

    def __init__(self, m):
        self.m = m

    def tensor_scale(self, amax, dtype):
        return float(OQ.nvfp4_tensor_scale(np.float32(amax.item()), "bf16"))

    def encode(self, hidden, ts):
        p, s, _ = OQ.quantize_nvfp4(hidden.to(torch.float32).numpy(), "bf16", ts=ts)
        return [torch.from_numpy(p), torch.from_numpy(s)]

    def experts(self, payload, local_ids, weights, ts, my_experts, pairs_hint=None):
        p, s = (t.numpy() for t in payload)
        lid = local_ids.numpy()
        w = weights.to(torch.float32).numpy()
        n, k = lid.shape
        H = self.m.down_proj.shape[1]
        rows = {}
        for le in np.unique(lid):
            if le >= len(my_experts):
                continue
            rr, jj = np.nonzero(lid == le)
            e = int(my_experts[le])
            gu = nvfp4_gemm(p[rr], s[rr], ts, self.m.gate_up_proj[e], self.m.gate_up_proj_scale[e],
                            self.m.gate_up_proj_scale_2)
            d = nvfp4_linear(OM.geglu(gu), self.m.down_proj[e], self.m.down_proj_scale[e], self.m.down_proj_scale_2)
            d = N.bf16(d * w[rr, jj][:, None])
            for i, (a, b) in enumerate(zip(rr, jj)):
                rows[(int(a), int(b))] = (le, d[i])
        out = np.zeros((n, H), np.float32)
        for a in range(n):
            part = np.zeros(H, np.float32)
            for le, d in sorted((v for (a2, _), v in rows.items() if a2 == a), key=lambda x: x[0]):
                part = N.bf16(part + d)
            out[a] = part
        return torch.from_numpy(out)

    def fold(self, rows, slot_row, T, world):
        rows = rows.numpy()
        sr = slot_row.numpy()
        H = self.m.down_proj.shape[1]
        out = np.zeros((T, H), np.float32)
        for t in range(T):
            for r in range(world):
                if sr[t, r] >= 0:
                    out[t] = N.bf16(out[t] + rows[sr[t, r]])
        return torch.from_numpy(out)


def main():
    rank, world, port, out_path, case = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], int(sys.argv[5])
    dense = len(sys.argv) > 6 and sys.argv[6] == "dense"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = port
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from aeo_quant_b200.bridges.gemma4.expert_parallel import balanced_placement, ep_moe_forward
    m, hidden, ids, w = case_inputs(case)
    E = m.num_experts
    T = hidden.shape[0]
    lo, hi = rank * T // world, (rank + 1) * T // world
    ops = OracleEpOps(m)
    owner = None
    if case == 2:
        load = np.bincount(ids[(ids >= 0) & (ids < E)], minlength=E)
        owner = balanced_placement(torch.from_numpy(load), world)
    y = ep_moe_forward(torch.from_numpy(hidden[lo:hi]).to(torch.bfloat16), torch.from_numpy(ids[lo:hi]),
                       torch.from_numpy(w[lo:hi]).to(torch.bfloat16), num_experts=E, group=None, ops=ops,
                       owner=owner, equal_tokens=dense)
    np.savez(out_path, y=y.numpy(), lo=lo, hi=hi)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
