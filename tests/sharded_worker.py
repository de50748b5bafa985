"""One rank of the 2-GPU sharded stack test (launched by test_multi_gpu.py through
torch.distributed.run): builds this rank's expert block, connects to the peer, decodes a
3-layer stack in both summation orders and saves the outputs for the parent test."""
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    torch.cuda.set_device(local)
    L, E, dim, ff, k = 3, 16, 2048, 512, 4
    rng = np.random.default_rng(77)
    x0 = rng.standard_normal(dim).astype(np.float32)
    logits = rng.standard_normal((2, L, E)).astype(np.float32)
    res = {}
    for exact in (False, True):
        b = ShardedBank(n_layers=L, n_experts=E, dim=dim, ff=ff, max_picks=k, device=local, rank=rank, world=world,
                        exact_order=exact)
        b.fill_synthetic(4242, 2)
        dist.barrier()
        outs = []
        for t in range(2):  # two tokens back to back: the exchange slots alternate
            outs.append(b.stack_decode(0, L, x0 if t == 0 else outs[-1], logits[t]))
        # device entry point, same tokens
        d_x = torch.from_numpy(x0.copy()).cuda()
        for t in range(2):
            d_l = torch.from_numpy(np.ascontiguousarray(logits[t])).cuda()
            torch.cuda.synchronize()
            b.stack_decode_device(0, L, d_x, d_l)
            b.synchronize()
        res[f"host_{int(exact)}"] = np.stack(outs)
        res[f"dev_{int(exact)}"] = d_x.cpu().numpy()
        dist.barrier()
        b.close()
    np.savez(os.path.join(a.out, f"rank{rank}.npz"), x0=x0, logits=logits, **res)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
