"""Failure detection without a GPU fault: a peer GPU that never posts its expert rows.

Rank 1 of a 2-rank expert-ID-sharded bank connects and then never decodes; rank 0
decodes with a short wait limit (clb_bank_set_wait_limit). Its stack kernel's bounded waits
for rank 1's rows run out, the kernel returns on its own, the call fails with CLB_E_CUDA and
the bank is poisoned (the next call fails with CLB_E_STATE). Only rank 0 ever runs a
kernel, so nothing waits on a kernel of another process. With fewer than 2 GPUs both
ranks' banks live on GPU 0 (two processes, one CUDA IPC mapping)."""
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
def test_peer_that_never_posts(cuda, tmp_path):
    import crosslane_b200 as cb
    torch = cuda
    same = torch.cuda.device_count() < 2
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(HERE, "timeout_worker.py"), "--out", str(tmp_path)] + (["--same-device"] if same else [])
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    with open(tmp_path / "rank0.json") as f:
        res = json.load(f)
    assert res["first"] == cb._capi.CLB_E_CUDA, res
    assert "bounded wait" in res["first_msg"]
    assert res["second"] == cb._capi.CLB_E_STATE, res
    assert res["seconds"] < 60, res  # the waits gave up on their own
