"""Host side of expert-ID sharding, on CPU: the expert blocks, the handle exchange over a
gloo process group, and the sharded combine (each rank computes the picks it owns, the
rows are gathered, every rank combines in ascending expert order) against the one-process
layer of the oracle, bit for bit."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, ".."))

from crosslane_b200 import sharded  # noqa: E402


@pytest.mark.parametrize("E,world", [(384, 8), (384, 2), (16, 3), (10, 4), (5, 5)])
def test_shard_blocks_cover_experts(E, world):
    seen = []
    for r in range(world):
        b, e = sharded.shard_range(E, r, world)
        assert b <= e
        seen.extend(range(b, e))
        for x in range(b, e):
            assert sharded.owner_of(x, E, world) == r
    assert seen == list(range(E))


def _worker(rank, world, port, out):
    import torch.distributed as dist
    from datetime import timedelta
    sys.path.insert(0, HERE)
    from oracle_lib import Oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # handle exchange: rank-indexed
        hs = sharded.exchange_handles(bytes([rank]) * 64)
        assert [h[0] for h in hs] == list(range(world))
        # sharded layer: own picks only, gather, combine everywhere
        orc = Oracle()
        E, dim, ff, k, seed = 12, 512, 256, 5, 99
        rng = np.random.default_rng(5)
        x = rng.standard_normal(dim).astype(np.float32)
        ids, w = orc.route_sigmoid(rng.standard_normal(E).astype(np.float32), k)
        b, e = sharded.shard_range(E, rank, world)
        mine = np.zeros((k, dim), np.float32)
        for p, ex in enumerate(ids):
            if b <= ex < e:
                t = orc.expert_type(2, seed, 0, int(ex))
                mats = [orc.synth_matrix(t, seed, 0, int(ex), role, n, kk)
                        for role, n, kk in ((0, ff, dim), (1, ff, dim), (2, dim, ff))]
                mine[p] = orc.expert(t, *mats, x, dim, ff)[1]
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        rows = np.sum(np.stack(parts), axis=0, dtype=np.float32)  # one owner per pick: exact
        got = orc.combine(ids, w, rows)  # every rank: ascending expert id fma chain
        want = orc.layer_synth(2, seed, 0, ids, w, x, dim, ff)
        np.save(os.path.join(out, f"r{rank}.npy"), np.stack([got, want]))
    finally:
        dist.destroy_process_group()


def test_sharded_combine_gloo(tmp_path):
    world = 2
    port = 29000 + os.getpid() % 1000
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        got, want = np.load(tmp_path / f"r{r}.npy")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _batch_worker(rank, world, port, out):
    """Batched exchange: every rank fills the expert rows of the picks it owns into a
    [T*k][dim] buffer (zeros elsewhere, including a -0.0 row value), an all-reduce (sum)
    over gloo gives every rank every row, and the per-token combine matches the
    one-process oracle layer bit for bit."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    sys.path.insert(0, HERE)
    from oracle_lib import Oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        orc = Oracle()
        E, dim, ff, k, T, seed = 10, 512, 256, 3, 4, 17
        rng = np.random.default_rng(8)
        xs = rng.standard_normal((T, dim)).astype(np.float32)
        routes = [orc.route_sigmoid(rng.standard_normal(E).astype(np.float32), k) for _ in range(T)]
        b, e = sharded.shard_range(E, rank, world)
        rows = np.zeros((T * k, dim), np.float32)
        for t, (ids, _) in enumerate(routes):
            for p, ex in enumerate(ids):
                if b <= ex < e:
                    ty = orc.expert_type(2, seed, 0, int(ex))
                    mats = [orc.synth_matrix(ty, seed, 0, int(ex), role, n, kk)
                            for role, n, kk in ((0, ff, dim), (1, ff, dim), (2, dim, ff))]
                    rows[t * k + p] = orc.expert(ty, *mats, xs[t], dim, ff)[1]
        buf = torch.from_numpy(rows.copy())
        dist.all_reduce(buf)
        got_rows = buf.numpy()
        got = np.stack([orc.combine(ids, w, got_rows[t * k:(t + 1) * k]) for t, (ids, w) in enumerate(routes)])
        want = np.stack([orc.layer_synth(2, seed, 0, ids, w, xs[t], dim, ff) for t, (ids, w) in enumerate(routes)])
        np.save(os.path.join(out, f"b{rank}.npy"), np.stack([got, want]))
        # the sum turns a -0.0 row value into +0.0; the combine's fma chain starts at +0.0,
        # so the combined output is the same either way
        ids, w = routes[0]
        r = got_rows[:k].copy()
        r[:, :8] = 0.0
        rn = r.copy()
        rn[:, :8] = -0.0
        assert np.array_equal(orc.combine(ids, w, r).view(np.uint32), orc.combine(ids, w, rn).view(np.uint32))
    finally:
        dist.destroy_process_group()


def test_sharded_batch_rows_allreduce_gloo(tmp_path):
    world = 2
    port = 30000 + os.getpid() % 1000
    mp.start_processes(_batch_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        got, want = np.load(tmp_path / f"b{r}.npy")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
