"""The config-5 workload of bench.py (--skewed): router logits = log Zipf(1.1) of each expert's
rank under a per-layer seeded permutation + Gumbel noise, so the top-6 is a draw of 6
distinct experts with Zipf probabilities. Checked on CPU against the workload's published
statistics: about 132 distinct experts per layer at batch 64 (5-95 % range 121-143), the
hottest rank picked far more often than a uniform draw, and layers permuted differently."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def top_k(logits, k=6):
    return np.argsort(-logits, axis=-1, kind="stable")[..., :k]


def test_distinct_experts_per_layer():
    rng = np.random.default_rng(0)
    lg = bench.zipf_logits(rng, 40, 64, 384)
    distinct = [len(np.unique(top_k(lg[l]))) for l in range(40)]
    assert 121 <= np.median(distinct) <= 143, np.median(distinct)
    assert 110 <= min(distinct) and max(distinct) <= 155, (min(distinct), max(distinct))


def test_rank_frequencies_follow_zipf():
    rng = np.random.default_rng(1)
    L, T, E = 2, 4000, 384
    lg = bench.zipf_logits(rng, L, T, E)
    perm_rank = [np.argsort(np.random.default_rng(bench.SEED + 7919 * l).permutation(E)) for l in range(L)]
    for l in range(L):
        counts = np.bincount(perm_rank[l][top_k(lg[l]).ravel()], minlength=E) / T  # by rank
        assert counts[0] > 0.7, counts[0]  # the hottest rank is in most tokens' top-6 (uniform: 6/384)
        assert counts[0] >= counts[9] >= counts[99]
        assert counts[200:].mean() < 0.01
    assert not np.array_equal(perm_rank[0], perm_rank[1])  # a different permutation per layer


def test_logits_pick_distinct_experts():
    rng = np.random.default_rng(2)
    lg = bench.zipf_logits(rng, 3, 50, 384)
    for l in range(3):
        for t in range(50):
            assert len(set(top_k(lg[l, t]).tolist())) == 6


def test_shard_load_matches_contiguous_blocks():
    """bench.shard_load uses the same contiguous expert blocks as sharded.shard_range, and at
    8 GPUs the Zipf workload's max/mean load (distinct experts decoded per GPU) is near the
    published 1.28."""
    from crosslane_b200 import sharded
    E = 384
    for world in (2, 3, 8):
        for e in range(E):
            b, end = sharded.shard_range(E, sharded.owner_of(e, E, world), world)
            assert b <= e < end and min((e * world) // E, world - 1) == sharded.owner_of(e, E, world)
    rng = np.random.default_rng(4)
    lg = bench.zipf_logits(rng, 40, 64, E)
    ratio = bench.shard_load([top_k(lg[l]) for l in range(40)], E, 8)
    assert 1.2 <= ratio <= 1.4, ratio
    assert bench.shard_load([top_k(lg[l]) for l in range(40)], E, 1) == 1.0
