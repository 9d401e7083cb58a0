"""Expert-parallel NVFP4 layer on 2 GPUs (NCCL all-to-all dispatch and
combine) equals the one-GPU grouped forward bit for bit."""
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
    y = torch.cat([r0["y"], r1["y"]])
    assert torch.equal(y.view(torch.int16), r0["ref"].view(torch.int16))
