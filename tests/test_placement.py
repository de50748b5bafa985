"""Frozen warm placement with the CUDA lane (STRATA_WARM_PLACEMENT_V1,
frozen_placement.hpp:5-16): the library's parser applies the reference's checks, the
Python writer round-trips, the greedy first placement honours capacity, and the cost
document has the schema crosslane's optimiser (rebalance.py:22-29) requires. GPU: a bank
holds exactly the experts placed on its lane and warm_execute matches the oracle with the
rest on the host lane."""
import numpy as np
import pytest

import crosslane_b200 as cb
from crosslane_b200 import placement as pl


def doc(nl=2, ne=4, tag=7, lanes=None):
    lanes = np.arange(nl * ne).reshape(nl, ne) % 4 if lanes is None else lanes
    return pl.format_placement(lanes, tag), lanes


def test_round_trip():
    text, lanes = doc()
    got, tag = pl.parse(text, 2, 4)
    assert tag == 7 and np.array_equal(got, lanes)
    assert text.splitlines()[0] == "STRATA_WARM_PLACEMENT_V1 2 4 7"


@pytest.mark.parametrize("mutate", [
    lambda t: t.replace("STRATA_WARM_PLACEMENT_V1", "STRATA_WARM_PLACEMENT_V2"),  # version
    lambda t: t.replace(" 2 4 7", " 3 4 7", 1),                                  # layer count
    lambda t: t.replace("\n0 1 ", "\n0 2 ", 1),                                  # unsorted / duplicate
    lambda t: t.rsplit("\n", 2)[0] + "\n",                                      # missing row
    lambda t: t + "1 3 0\n",                                                     # extra row
    lambda t: t + "junk",                                                        # trailing data
    lambda t: t.replace("\n1 2 2", "\n1 2 4", 1),                                # lane out of range
    lambda t: t.replace("\n0 0 0", "\n0 0 -1", 1),                               # negative lane
    lambda t: t.replace("\n0 3 3", "\n0 3 x", 1),                                # not a number
])
def test_rejects(mutate):
    text, _ = doc()
    bad = mutate(text)
    assert bad != text
    with pytest.raises(cb.ClbError) as ei:
        pl.parse(bad, 2, 4)
    assert ei.value.code == 1 and "placement" in str(ei.value)


def test_greedy_respects_capacity_and_floor():
    rng = np.random.default_rng(0)
    counts = rng.integers(0, 100, (3, 8))
    nbytes = rng.integers(10, 20, (3, 8))
    cap = int(nbytes.sum() // 3)
    lanes = pl.greedy(counts, nbytes, cap, floor_per_layer=1)
    assert int(nbytes[lanes == pl.CUDA].sum()) <= cap
    for l in range(3):  # every layer keeps its hottest expert on the lane
        assert lanes[l, int(np.argmax(counts[l]))] == pl.CUDA or counts[l].max() == 0
    assert np.array_equal(lanes, pl.greedy(counts, nbytes, cap, floor_per_layer=1))  # deterministic


def test_rebalance_cost_document():
    d = pl.rebalance_costs({0: 100.0, 1: 120.0}, {0: 900.0, 1: 950.0}, 64, b"profile", gpu_slot="hip")
    assert d["schema"] == "strata-warm-costs-v1" and d["scope"] == "measured-decode-excluding-warmup"
    assert d["decode_tokens"] == 64 and len(d["layers"]) == 2
    assert all(set(r) == {"cpu", "hip", "sycl"} and r["hip"]["per_expert_ns"] > 0 for r in d["layers"])
    with pytest.raises(ValueError):
        pl.rebalance_costs({0: 1.0}, {1: 1.0}, 1, b"")


@pytest.mark.gpu
def test_bank_holds_placed_experts(cuda, orc):
    nl, ne, dim, ff, seed, policy = 2, 12, 2048, 512, 4, 2
    lanes = np.zeros((nl, ne), np.int32)
    lanes[0, [1, 3, 5, 7]] = pl.CUDA
    lanes[1, [0, 2, 9]] = pl.CUDA
    lanes[1, 4] = pl.SYCL
    placed, _ = pl.parse(pl.format_placement(lanes, 1), nl, ne)
    bank = cb.ExpertBank(n_layers=nl, n_experts=ne, dim=dim, ff=ff, max_picks=6, device=0)
    try:
        bank.apply_placement(placed, pl.CUDA)
        bank.fill_synthetic(seed, policy)
        for l in range(nl):
            for e in range(ne):
                assert bank.warm_contains(l, e) == (lanes[l, e] == pl.CUDA)
        with pytest.raises(cb.ClbError):  # weights loaded: placement is frozen
            bank.apply_placement(placed, pl.CUDA)
        rng = np.random.default_rng(1)
        ids = np.array([1, 2, 3, 8], np.int32)  # 1, 3 on the CUDA lane; 2, 8 on the host lane
        w = np.array([0.4, 0.3, 0.2, 0.1], np.float32)
        x = rng.standard_normal(dim).astype(np.float32)

        def host_lane(layer, expert, xv):
            return orc.layer_synth(policy, seed, layer, np.array([expert], np.int32), np.array([1.0], np.float32),
                                   xv, dim, ff)

        got = bank.warm_execute(0, ids, w, x, host_lane=host_lane)
        want = orc.layer_synth(policy, seed, 0, ids, w, x, dim, ff)
        from oracle_lib import rel_l2
        assert rel_l2(got, want) <= 1e-3
    finally:
        bank.close()


def _reference_rebalance(request):
    """crosslane's own optimiser module (engine/strata/warm/rebalance.py), loaded from the
    checkout the tests compile against; skipped where no checkout exists."""
    import importlib.util
    import os
    ref = request.config.getoption("--crosslane-ref") or os.environ.get("CROSSLANE_REF")
    recorded = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "checkout")
    if not ref and os.path.isfile(recorded):
        with open(recorded) as f:
            ref = f.read().strip()
    path = os.path.join(ref or "", "engine", "strata", "warm", "rebalance.py")
    if not ref or not os.path.isfile(path):
        pytest.skip("no crosslane checkout (set CROSSLANE_REF or --crosslane-ref)")
    spec = importlib.util.spec_from_file_location("crosslane_rebalance", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _plan_and_profile(tmp_path, counts, hip_room, sycl_room, hip_resident, sycl_members):
    """A two-layer, four-expert plan in the shape crosslane's native planner writes (the
    fields rebalance.py:25-52 reads) and the decode profile of selection counts."""
    profile = tmp_path / "decode.bin"
    profile.write_bytes(b"".join(int(c).to_bytes(4, "little") for c in counts))
    g = 2 ** 21
    plan = {"layers": 2, "sycl_footprint": 1_000_000_000, "hip_footprint": 1_000_000_000,
            "warm_inventory": [[l, e, g, g, "IQ2_XXS", "IQ2_XS", "IQ1_M"] for l in range(2) for e in range(4)],
            "hip_resident": {"experts": [[l, e, 0, g] for l, e in hip_resident]},
            "warm_sycl": {"members": [[l, e] for l, e in sycl_members], "reservation_bytes": sycl_room,
                          "profile_tag": 7},
            "warm_hip_room_bytes": hip_room}
    return plan, profile


def test_reference_optimiser_accepts_cuda_costs_in_hip_slot(request, tmp_path):
    """The CUDA lane in the HIP column next to a measured B65 lane: crosslane's optimiser
    accepts the cost document and moves the hot CPU experts onto the CUDA lane."""
    rb = _reference_rebalance(request)
    counts = [1, 1, 10, 0] * 2  # expert 2 of each layer is hot and starts on the CPU lane
    plan, profile = _plan_and_profile(tmp_path, counts, hip_room=2 * 2 ** 21, sycl_room=2 * 2 ** 21,
                                      hip_resident=[(0, 0), (1, 0)], sycl_members=[(0, 1), (1, 1)])
    costs = pl.rebalance_costs({0: 1.0, 1: 1.0}, {0: 10.0, 1: 10.0}, 12, profile.read_bytes(), gpu_slot="hip",
                               other_ns={0: 2.0, 1: 2.0})
    assigned, report = rb.optimise(plan, str(profile), costs, min_payload=0)
    assert report["after_ns"] < report["before_ns"]
    assert all(assigned[l, 2] == pl.HIP for l in range(2))  # the CUDA lane holds the GPU slot 1
    text = rb.assignment_text(assigned, plan)
    lanes, tag = pl.parse(text, 2, 4)  # the optimiser's output is a document this library applies
    assert tag == 7 and lanes[0, 2] == pl.HIP


def test_reference_optimiser_with_lone_cuda_lane(request, tmp_path):
    """The CUDA lane alone, in the SYCL column (the one with the optimiser's per-layer
    coverage floor); the unused HIP column has no room, so nothing can land there."""
    rb = _reference_rebalance(request)
    counts = [1, 10, 1, 0] * 2
    plan, profile = _plan_and_profile(tmp_path, counts, hip_room=0, sycl_room=2 * 2 ** 21, hip_resident=[],
                                      sycl_members=[(0, 0), (1, 0)])
    costs = pl.rebalance_costs({0: 1.0, 1: 1.0}, {0: 10.0, 1: 10.0}, 12, profile.read_bytes(), gpu_slot="sycl")
    assert all(r["hip"]["measurement_source"].startswith("unused") for r in costs["layers"])
    assigned, report = rb.optimise(plan, str(profile), costs, min_payload=0)
    assert report["after_ns"] < report["before_ns"]
    assert all(assigned[l, 1] == pl.SYCL for l in range(2))  # the hot expert moved onto the CUDA lane
    assert all(lane != pl.HIP for lane in assigned.values())  # the lane without room got nothing
    bad = dict(costs, profile_sha256="0" * 64)  # provenance still enforced
    with pytest.raises(ValueError):
        rb.optimise(plan, str(profile), bad, min_payload=0)
