"""One rank of the 2-GPU sharded batched-stack test (launched by test_multi_gpu.py through
torch.distributed.run, NCCL process group): this rank's expert block decodes a batch of
tokens through 2 layers with the per-layer row exchange (all-reduce of the expert rows),
and rank 0 also runs the unsharded batched stack on a full bank; outputs are saved for the
parent test."""
import argparse
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
import crosslane_b200 as cb  # noqa: E402
from crosslane_b200.sharded import ShardedBank  # noqa: E402

L, E, DIM, FF, K, T, SEED = 2, 24, 1024, 512, 6, 40, 606


def zipf_logits(rng, layers, tokens, experts, s=1.1):
    logp = -s * np.log(np.arange(1, experts + 1, dtype=np.float64))
    out = np.empty((layers, tokens, experts), np.float32)
    for l in range(layers):
        rank_of = np.argsort(rng.permutation(experts))
        out[l] = (logp[rank_of][None, :] + rng.gumbel(size=(tokens, experts))).astype(np.float32)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rng = np.random.default_rng(31)
    h0 = rng.standard_normal((T, DIM)).astype(np.float32)
    logits = zipf_logits(rng, L, T, E)
    b = ShardedBank(n_layers=L, n_experts=E, dim=DIM, ff=FF, max_picks=K, device=local, rank=rank, world=world)
    b.fill_synthetic(SEED, 2)
    d_h = torch.from_numpy(h0.copy()).cuda()
    d_lg = torch.from_numpy(logits).cuda()
    d_ws = torch.zeros(b.stack_batch_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    d_rows = torch.zeros((T * K, DIM), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    b.stack_batch_device(0, L, d_h, d_lg, d_ws, d_rows)
    b.synchronize()
    res = {"sharded": d_h.cpu().numpy(), "h0": h0, "logits": logits}
    dist.barrier()
    del d_h, d_ws, d_rows  # used on the bank stream: freed before the bank destroys it
    torch.cuda.synchronize()
    b.close()
    if rank == 0:  # the same batch on one full bank
        f = cb.ExpertBank(n_layers=L, n_experts=E, dim=DIM, ff=FF, max_picks=K, device=local)
        f.fill_synthetic(SEED, 2)
        d_f = torch.from_numpy(h0.copy()).cuda()
        d_wf = torch.zeros(f.stack_batch_workspace_bytes(T), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        f.stack_batch_device(0, L, d_f, d_lg, d_wf)
        f.synchronize()
        res["single"] = d_f.cpu().numpy()
        del d_f, d_wf
        torch.cuda.synchronize()
        f.close()
    np.savez(os.path.join(a.out, f"batch_rank{rank}.npz"), **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
