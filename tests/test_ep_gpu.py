"""Expert-parallel NVFP4 layer on 2 GPUs (NCCL all-to-all dispatch and
combine) against the one-GPU grouped forward."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_match_one_gpu(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = str(s.getsockname()[1])
    outs = [str(tmp_path / f"r{r}.pt") for r in range(2)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "ep_gpu_worker.py"), str(r), "2", port, outs[r]],
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, env=env) for r in range(2)]
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=300)[0].decode(errors="replace"))
        except subprocess.TimeoutExpired:
            p.kill()
            pytest.fail("expert-parallel GPU worker timed out")
    assert all(p.returncode == 0 for p in procs), "\n".join(logs)
    r0, r1 = (torch.load(o) for o in outs)
    y = torch.cat([r0["y"], r1["y"]]).float().numpy()
    ref = r0["ref"].float().numpy()
    # The expert-parallel layer folds each rank's experts first, then the
    # ranks' partial rows: only the association of the bf16 fold differs
    # from one GPU, so every output is within 2e-3 * max|ref| or k bf16 ulps
    # of the token's largest weighted expert output (from the oracle).
    sys.path.insert(0, HERE)
    import numpy as np
    from ep_worker import pair_outputs
    from helpers import TOL, bf16_ulp
    from oracle import moe as OM
    inp = r0["inputs"]
    gp, gs, gt, dp, ds, dt = (t.numpy() for t in inp["weights"])
    m = OM.NVFP4Experts(gp, gs, float(gt), dp, ds, float(dt))
    ids = inp["ids"].numpy()
    hid = inp["hid"].float().numpy()
    pairs = pair_outputs(m, hid, ids, inp["w"].float().numpy())
    big = np.zeros(hid.shape[0], np.float32)
    for (t, _), row in pairs.items():
        big[t] = max(big[t], float(np.abs(row).max()))
    lim = np.maximum(TOL * np.abs(ref).max(), ids.shape[1] * bf16_ulp(big)[:, None])
    assert np.all(np.abs(y.astype(np.float64) - ref) <= lim)
    # the fixed-size, host-sync-free dispatch gives the same bits
    assert torch.equal(torch.cat([r0["y_dense"], r1["y_dense"]]), torch.cat([r0["y"], r1["y"]]))
    # the C-ABI layer (dispatch, experts, combine over its own NCCL
    # communicator) gives the Python layer's bits
    assert torch.equal(torch.cat([r0["y_capi"], r1["y_capi"]]), torch.cat([r0["y"], r1["y"]]))
