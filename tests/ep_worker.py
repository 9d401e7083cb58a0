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


class OracleEpOps:
    """Oracle arithmetic for ep_moe_forward (the rank's experts only)."""

    def __init__(self, m, first, count):
        self.m, self.first, self.count = m, first, count

    def tensor_scale(self, amax, dtype):
        return float(OQ.nvfp4_tensor_scale(np.float32(amax.item()), "bf16"))

    def encode(self, hidden, ts):
        p, s, _ = OQ.quantize_nvfp4(hidden.to(torch.float32).numpy(), "bf16", ts=ts)
        return [torch.from_numpy(p), torch.from_numpy(s)]

    def experts(self, payload, local_ids, weights, ts, my_experts):
        p, s = (t.numpy() for t in payload)
        lid = local_ids.numpy()
        w = weights.to(torch.float32).numpy()
        H = self.m.down_proj.shape[1]
        out = np.zeros((p.shape[0], H), np.float32)
        for le in np.unique(lid):
            rows = np.nonzero(lid == le)[0]
            e = int(my_experts[le])
            gu = nvfp4_gemm(p[rows], s[rows], ts, self.m.gate_up_proj[e], self.m.gate_up_proj_scale[e],
                            self.m.gate_up_proj_scale_2)
            d = nvfp4_linear(OM.geglu(gu), self.m.down_proj[e], self.m.down_proj_scale[e], self.m.down_proj_scale_2)
            out[rows] = N.bf16(d * w[rows][:, None])
        return torch.from_numpy(out)

    def combine(self, rows, pair_row, top_k_index, T, k):
        rows = rows.numpy()
        pr = pair_row.numpy()
        ids = top_k_index.numpy()
        out = np.zeros((T, rows.shape[1] if rows.ndim == 2 else self.m.down_proj.shape[1]), np.float32)
        for t in range(T):
            for j in np.argsort(ids[t], kind="stable"):
                r = pr[t * k + j]
                if r >= 0:
                    out[t] = N.bf16(out[t] + rows[r])
        return torch.from_numpy(out)


def main():
    rank, world, port, out_path, case = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], int(sys.argv[5])
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = port
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from aeo_quant_b200.bridges.gemma4.expert_parallel import balanced_placement, ep_moe_forward
    m, hidden, ids, w = case_inputs(case)
    E = m.num_experts
    T = hidden.shape[0]
    lo, hi = rank * T // world, (rank + 1) * T // world
    e_loc = E // world
    ops = OracleEpOps(m, rank * e_loc, e_loc)
    owner = None
    if case == 2:
        load = np.bincount(ids[(ids >= 0) & (ids < E)], minlength=E)
        owner = balanced_placement(torch.from_numpy(load), world)
    y = ep_moe_forward(torch.from_numpy(hidden[lo:hi]).to(torch.bfloat16), torch.from_numpy(ids[lo:hi]),
                       torch.from_numpy(w[lo:hi]).to(torch.bfloat16), num_experts=E, group=None, ops=ops,
                       owner=owner)
    np.savez(out_path, y=y.numpy(), lo=lo, hi=hi)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
