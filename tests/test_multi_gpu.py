"""Expert-ID sharding over 2 GPUs (persistent stack kernel with peer-store exchange).
Skipped on machines with fewer than 2 GPUs."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle_lib import bits, rel_l2

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.gpu
def test_sharded_stack_two_gpus(orc, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29533",
           os.path.join(HERE, "sharded_worker.py"), "--out", str(tmp_path)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    d0, d1 = (np.load(tmp_path / f"rank{i}.npz") for i in range(2))
    L, E, dim, ff, k = 3, 16, 2048, 512, 4
    for key in ("host_0", "host_1", "dev_0", "dev_1"):
        assert np.array_equal(bits(d0[key]), bits(d1[key])), key  # every GPU holds the same residual stream
    x0, logits = d0["x0"], d0["logits"]
    # exact order: bit-identical to the single-device oracle, token after token
    h = x0
    for t in range(2):
        h = orc.stack(2, 4242, h, logits[t], dim, ff, k=k)
        assert np.array_equal(bits(d0["host_1"][t]), bits(h)), f"token {t}"
    # fast order: within the drift bound of the unsharded stack
    want = orc.stack(2, 4242, x0, logits[0], dim, ff, k=k)
    bound = max(1e-3, 4 * orc.stack_sensitivity(2, 4242, x0, logits[0], dim, ff, k))
    assert rel_l2(d0["host_0"][0], want) <= bound


@pytest.mark.gpu
def test_sharded_batched_stack_two_gpus(orc, tmp_path):
    """Batched stack sharded by expert ID over 2 GPUs (per-layer all-reduce of the expert
    rows over NCCL): both GPUs hold the same residual streams, bit-identical to the
    unsharded batched stack on one GPU, and within the stack's drift bound of the oracle."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(HERE, "sharded_batch_worker.py"), "--out", str(tmp_path)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    d0, d1 = (np.load(tmp_path / f"batch_rank{i}.npz") for i in range(2))
    assert np.array_equal(bits(d0["sharded"]), bits(d1["sharded"]))
    assert np.array_equal(bits(d0["sharded"]), bits(d0["single"])), "sharded differs from one GPU"
    h0, logits = d0["h0"], d0["logits"]
    dim, ff, k, seed = 1024, 512, 6, 606
    ratios = []
    for t in range(0, h0.shape[0], 7):
        want = orc.stack(2, seed, h0[t], logits[:, t, :], dim, ff, k)
        bound = max(1e-3, 4 * orc.stack_sensitivity(2, seed, h0[t], logits[:, t, :], dim, ff, k))
        ratios.append(rel_l2(d0["sharded"][t], want) / bound)
    assert np.median(ratios) <= 1.0, ratios  # the free-running stack: drift bound for the median token
