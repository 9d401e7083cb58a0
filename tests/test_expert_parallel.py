"""Expert-parallel dispatch/combine: two gloo ranks on CPU run the shared
orchestration with oracle arithmetic; their outputs must equal, bit for
bit, the expert-parallel fold order restated on one process, and lie within
the output tolerance of the one-process oracle prefill forward."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import moe as OM

from helpers import TOL, bf16_ulp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return str(s.getsockname()[1])


@pytest.mark.parametrize("case,mode", [(0, "compact"), (1, "compact"), (2, "compact"), (3, "compact"),
                                       (0, "dense"), (2, "dense")])
def test_ep_two_ranks_match_one_process(tmp_path, case, mode):
    sys.path.insert(0, HERE)
    from ep_worker import case_inputs
    world, port = 2, _free_port()
    outs = [str(tmp_path / f"r{r}.npz") for r in range(world)]
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_worker.py"), str(r), str(world), port,
                               outs[r], str(case), mode], stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
             for r in range(world)]
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=240)[0].decode(errors="replace"))
        except subprocess.TimeoutExpired:
            p.kill()
            pytest.fail("expert-parallel worker timed out")
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)
    from ep_worker import ep_order_reference
    from aeo_quant_b200.bridges.gemma4.expert_parallel import balanced_placement, contiguous_placement
    m, hidden, ids, w = case_inputs(case)
    y = np.zeros((hidden.shape[0], m.down_proj.shape[1]), np.float32)
    for o in outs:
        d = np.load(o)
        y[int(d["lo"]):int(d["hi"])] = d["y"]
    E = m.num_experts
    if case == 2:
        owner = balanced_placement(torch.from_numpy(np.bincount(ids[(ids >= 0) & (ids < E)], minlength=E)), world)
    else:
        owner = contiguous_placement(E, world)
    # bit for bit the expert-parallel fold order restated on one process ...
    exp = ep_order_reference(m, hidden, ids, w, owner.numpy(), world)
    np.testing.assert_array_equal(y.view(np.uint32), exp.view(np.uint32))
    # ... and next to the one-GPU forward: the two differ only in the
    # association of the bf16 fold, so each output is within 2e-3 * max|ref|
    # or k bf16 ulps of the token's largest addend
    from ep_worker import pair_outputs
    ref = OM.nvfp4_prefill(m, hidden, ids, w)
    pairs = pair_outputs(m, hidden, ids, w)
    big = np.zeros(hidden.shape[0], np.float32)
    for (t, _), row in pairs.items():
        big[t] = max(big[t], float(np.abs(row).max()))
    lim = np.maximum(TOL * np.abs(ref).max(), ids.shape[1] * bf16_ulp(big)[:, None])
    assert np.all(np.abs(y.astype(np.float64) - ref) <= lim)


def test_plan_dispatch_groups_pairs_by_rank():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "aeo-quant_b200"))
    from aeo_quant_b200.bridges.gemma4.expert_parallel import plan_dispatch
    ids = torch.tensor([[7, 0, 4], [1, 8, 5]])          # E = 8, world = 2: experts 0-3 on rank 0
    send, counts, dest = plan_dispatch(ids, 8, 2)
    assert counts.tolist() == [2, 3]
    assert send.tolist() == [1, 3, 0, 2, 5]             # rank 0: pairs 1, 3; rank 1: pairs 0, 2, 5
    assert dest.tolist() == [1, 0, 1, 0, 2, 1]          # id 8 (== E) is dropped
    with pytest.raises(ValueError, match="divisible by the world size"):
        plan_dispatch(ids, 8, 3)


def test_balanced_placement_and_local_index():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "aeo-quant_b200"))
    from aeo_quant_b200.bridges.gemma4.expert_parallel import (balanced_placement, contiguous_placement,
                                                               local_index, plan_dispatch)
    # Zipf-like load over 16 experts, hot experts at the low ids
    load = torch.tensor([1.0 / (e + 1) ** 1.2 for e in range(16)])
    owner = balanced_placement(load, 4)
    assert torch.bincount(owner, minlength=4).tolist() == [4, 4, 4, 4]
    per_rank = torch.zeros(4, dtype=torch.float64).index_add_(0, owner, load.double())
    contig = torch.zeros(4, dtype=torch.float64).index_add_(0, contiguous_placement(16, 4), load.double())
    assert per_rank.max() < contig.max()
    # the hottest expert's rank is filled up with the coldest ones
    assert per_rank.max() <= load.double().max() + load.double().sort().values[:3].sum() + 1e-9
    assert owner[:4].tolist() == [0, 1, 2, 3]          # the four hottest go to different ranks
    local = local_index(owner, 4)
    for r in range(4):
        mine = torch.nonzero(owner == r).reshape(-1)
        assert local[mine].tolist() == list(range(4))
    ids = torch.tensor([[0, 5], [16, 1]])               # 16 == E: dropped
    send, counts, dest = plan_dispatch(ids, 16, 4, owner)
    assert dest.tolist() == [int(owner[0]), int(owner[5]), 4, int(owner[1])]
    assert counts.sum().item() == 3
    assert torch.equal(local_index(contiguous_placement(16, 4), 4), torch.arange(16) % 4)
    with pytest.raises(ValueError, match="every rank"):
        local_index(torch.zeros(16, dtype=torch.int64), 4)
    with pytest.raises(ValueError, match="divisible"):
        balanced_placement(load, 3)


def test_plan_token_dispatch_one_send_per_token_and_rank():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "aeo-quant_b200"))
    from aeo_quant_b200.bridges.gemma4.expert_parallel import plan_token_dispatch
    ids = torch.tensor([[7, 0, 4], [1, 8, 5], [2, 3, 1]])   # E = 8, world = 2: experts 0-3 on rank 0
    send_tok, send_dest, counts, lid = plan_token_dispatch(ids, 8, 2)
    assert counts.tolist() == [3, 2]
    assert list(zip(send_dest.tolist(), send_tok.tolist())) == [(0, 0), (0, 1), (0, 2), (1, 0), (1, 1)]
    # local ids on the destination, 4 (= E/world, dropped) where the slot lives elsewhere or is invalid
    assert lid.tolist() == [[4, 0, 4], [1, 4, 4], [2, 3, 1], [3, 4, 0], [4, 4, 1]]
    empty = plan_token_dispatch(torch.zeros(0, 3, dtype=torch.int64), 8, 2)
    assert empty[0].numel() == 0 and empty[2].tolist() == [0, 0]
