"""One rank of the bounded-wait failure test (launched by test_wait_timeout.py through
torch.distributed.run, host plumbing over gloo): rank 1 builds its expert block, connects
and then never decodes -- a peer that never posts its rows. Rank 0 decodes with a short
wait limit: its stack kernel's waits for rank 1's rows run out, the kernel returns, the call
fails with CLB_E_CUDA and the bank is poisoned (CLB_E_STATE afterwards). Rank 1 keeps its
bank (the memory rank 0 stores into) alive until rank 0 is done."""
import argparse
import json
import os
import sys
import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
import crosslane_b200 as cb  # noqa: E402
from crosslane_b200._capi import CLB_E_CUDA, CLB_E_STATE  # noqa: E402
from crosslane_b200.sharded import ShardedBank  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--same-device", action="store_true")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = 0 if a.same_device else int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    torch.cuda.set_device(device)
    L, E, dim, ff, k = 2, 16, 2048, 512, 4
    b = ShardedBank(n_layers=L, n_experts=E, dim=dim, ff=ff, max_picks=k, device=device, rank=rank, world=world)
    b.fill_synthetic(99, 2)
    dist.barrier()
    res = {"rank": rank}
    if rank == 0:
        b.set_wait_limit(1 << 14)
        rng = np.random.default_rng(5)
        x = rng.standard_normal(dim).astype(np.float32)
        logits = rng.standard_normal((L, E)).astype(np.float32)
        logits[:, E // 2:] += 10.0  # every pick in rank 1's block: rank 0 can only wait for its rows
        t0 = time.time()
        try:
            b.stack_decode(0, L, x, logits)
            res["first"] = "ok"
        except cb.ClbError as e:
            res["first"] = e.code
            res["first_msg"] = str(e)
        res["seconds"] = time.time() - t0
        try:
            b.stack_decode(0, L, x, logits)
            res["second"] = "ok"
        except cb.ClbError as e:
            res["second"] = e.code
        res["expect"] = [CLB_E_CUDA, CLB_E_STATE]
    dist.barrier()  # rank 1 stays (with its bank) until rank 0's kernel has returned
    with open(os.path.join(a.out, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    b.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
