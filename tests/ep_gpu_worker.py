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


def capi_layer(m, x, ids, w, E):
    """The same layer through the C ABI only: aeoq_ep_dispatch ->
    aeoq_ep_experts_nvfp4 -> aeoq_ep_combine over a communicator made by
    aeoq_ep_nccl_comm_init (the unique id travels over the process group, as
    a host would pass it)."""
    import ctypes
    from aeo_quant_b200 import _capi as A
    lib = A.load()
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = x.device
    n_id = lib.aeoq_ep_nccl_unique_id_bytes()
    buf = ctypes.create_string_buffer(n_id)
    if rank == 0:
        A.check(lib.aeoq_ep_nccl_unique_id(buf, n_id))
    uid = torch.frombuffer(bytearray(buf.raw), dtype=torch.uint8).to(dev)
    dist.broadcast(uid, 0)
    uid_host = ctypes.create_string_buffer(bytes(uid.cpu().numpy().tobytes()), n_id)
    comm = ctypes.c_void_p()
    A.check(lib.aeoq_ep_nccl_comm_init(ctypes.byref(comm), world, rank, uid_host))
    T, H = x.shape
    k = ids.shape[1]
    I = m.down_proj.shape[2] * 2
    e_loc = m.gate_up_proj.shape[0]
    x, ids, w = x.contiguous(), ids.contiguous(), w.to(torch.bfloat16).contiguous()
    u8, i32 = dict(dtype=torch.uint8, device=dev), dict(dtype=torch.int32, device=dev)
    n = world * T
    rp, rs = torch.empty(n, H // 2, **u8), torch.empty(n, H // 16, **u8)
    rl, rw = torch.empty(n, k, **i32), torch.empty(n, k, dtype=torch.bfloat16, device=dev)
    ts = torch.empty((), dtype=torch.bfloat16, device=dev)
    slot_row = torch.empty(T, world, **i32)
    st = A.stream_ptr(dev)
    ws = torch.empty(lib.aeoq_ep_dispatch_workspace_size(world, T, k, H), **u8)
    A.check(lib.aeoq_ep_dispatch(comm, world, rank, x.data_ptr(), T, H, ids.data_ptr(), A.dtype_code(ids.dtype),
                                 w.data_ptr(), k, E, None, rp.data_ptr(), rs.data_ptr(), rl.data_ptr(), rw.data_ptr(),
                                 ts.data_ptr(), slot_row.data_ptr(), ws.data_ptr(), ws.numel(), st))
    gu_atoms = A.weight_atoms(m.gate_up_proj_scale, e_loc, 2 * I, H, geglu_inter=I)
    dw_atoms = A.weight_atoms(m.down_proj_scale, e_loc, H, I)
    rows = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
    ws2 = torch.empty(lib.aeoq_ep_experts_nvfp4_workspace_size(n, k, T * k, e_loc, H, I), **u8)
    A.check(lib.aeoq_ep_experts_nvfp4(rp.data_ptr(), rs.data_ptr(), ts.data_ptr(), n, rl.data_ptr(), rw.data_ptr(), k,
                                      T * k, m.gate_up_proj.data_ptr(), gu_atoms.data_ptr(),
                                      m.gate_up_proj_scale_2.data_ptr(), A.dtype_code(m.gate_up_proj_scale_2.dtype),
                                      m.down_proj.data_ptr(), dw_atoms.data_ptr(), m.down_proj_scale_2.data_ptr(),
                                      A.dtype_code(m.down_proj_scale_2.dtype), e_loc, H, I, rows.data_ptr(),
                                      ws2.data_ptr(), ws2.numel(), A.err_word(dev).data_ptr(), st))
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ws3 = torch.empty(lib.aeoq_ep_combine_workspace_size(world, T, H), **u8)
    A.check(lib.aeoq_ep_combine(comm, world, rank, rows.data_ptr(), slot_row.data_ptr(), T, H, out.data_ptr(),
                                ws3.data_ptr(), ws3.numel(), st))
    torch.cuda.synchronize(dev)
    A.check(lib.aeoq_ep_nccl_comm_destroy(comm))
    return out.cpu()


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
    res = {"y": y.cpu(), "y_dense": y_dense.cpu(), "y_capi": capi_layer(m, hid[lo:hi], ids[lo:hi], w[lo:hi], E),
           "lo": lo, "hi": hi}
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
