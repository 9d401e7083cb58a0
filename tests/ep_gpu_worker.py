"""One rank of the 2-GPU expert-parallel test (NCCL): builds the same
16-expert NVFP4 layer on every rank, keeps its 8 experts, runs the
expert-parallel forward on its half of the tokens; rank 0 also runs the
one-GPU grouped forward over all tokens and saves the layer and inputs.
Launched by test_ep_gpu.py."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, ROOT, os.path.join(ROOT, "aeo-quant_b200")):
    sys.path.insert(0, p)

import types  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world, port, out_path = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = port
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from aeo_quant_b200.bridges.gemma4 import moe_ops
    from aeo_quant_b200.bridges.gemma4.expert_parallel import ExpertParallelNVFP4
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    from aeo_quant_b200.gpu import quant as Q
    dev = torch.device("cuda", rank)
    E, H, I, k, T = 16, 2816, 704, 8, 96
    g = torch.Generator().manual_seed(0)
    wgu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wd = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    hid = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(dev)
    ids[5, 3] = E                                          # a dropped id
    w = torch.softmax(torch.randn(T, k, generator=g), -1).to(torch.bfloat16).to(dev)
    gp, gs, gt = Q.quantize_3d_to_nvfp4(wgu)
    dp, ds, dt = Q.quantize_3d_to_nvfp4(wd)
    e_loc = E // world
    sl = slice(rank * e_loc, (rank + 1) * e_loc)
    cfg = types.SimpleNamespace(num_experts=e_loc, hidden_size=H, moe_intermediate_size=I,
                                hidden_activation="gelu_pytorch_tanh")
    m = Gemma4TextExpertsNVFP4(cfg).to(dev)
    m.gate_up_proj.copy_(gp[sl]); m.gate_up_proj_scale.copy_(gs[sl]); m.gate_up_proj_scale_2.copy_(gt.float())
    m.down_proj.copy_(dp[sl]); m.down_proj_scale.copy_(ds[sl]); m.down_proj_scale_2.copy_(dt.float())
    ep = ExpertParallelNVFP4(m, E)
    lo, hi = rank * T // world, (rank + 1) * T // world
    y = ep(hid[lo:hi], ids[lo:hi], w[lo:hi])
    ep.equal_tokens = True                                 # fixed-size all-to-alls, no host sync
    y_dense = ep(hid[lo:hi], ids[lo:hi], w[lo:hi])
    res = {"y": y.cpu(), "y_dense": y_dense.cpu(), "lo": lo, "hi": hi}
    if rank == 0:
        res["ref"] = moe_ops.nvfp4_experts_grouped(hid, ids, w, gp, gs, gt.float(), dp, ds, dt.float()).cpu()
        res["inputs"] = {"hid": hid.cpu(), "ids": ids.cpu(), "w": w.cpu(),
                         "weights": [t.cpu() for t in (gp, gs.view(torch.uint8), gt.float(), dp, ds.view(torch.uint8),
                                                       dt.float())]}
    torch.save(res, out_path)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
