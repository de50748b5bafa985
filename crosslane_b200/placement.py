"""Frozen warm placement and the rebalancer's cost document with this library as a lane.

crosslane freezes which lane serves each (layer, expert) in a STRATA_WARM_PLACEMENT_V1
document (engine/strata/warm/frozen_placement.hpp:5-16) and chooses it with a
critical-path optimiser over measured per-selection service costs
(engine/strata/warm/rebalance.py, costs from make_costs.py, schema
"strata-warm-costs-v1"). This module adds the CUDA lane to both:

* ``parse`` / ``format_placement``: the document, lanes 0 CPU, 1 HIP, 2 SYCL and
  ``CUDA`` = 3 (a document may equally give this lane the GPU slot 1); parsing goes through
  the library's ``clb_placement_parse`` so host and library apply the same checks;
* ``ExpertBank.apply_placement``: the bank holds exactly the experts placed on its lane;
  ``warm_execute`` sends every other pick to its host lane;
* ``measure_cuda_costs``: per-layer per-selection service ns of the CUDA lane, measured
  through the bank's batched entry point (issue overhead absorbed, as make_costs.py does);
* ``rebalance_costs``: a "strata-warm-costs-v1" document whose GPU column is the CUDA lane,
  so crosslane's own optimiser can place experts between the CPU lane and this one;
* ``greedy``: a capacity-bounded first placement (hottest experts per byte first) for
  when no measured profile exists yet.
"""
import ctypes as C
import hashlib
import time

import numpy as np

from ._capi import ErrorV1, check, lib

LANES = ("cpu", "hip", "sycl", "cuda")
CPU, HIP, SYCL, CUDA = 0, 1, 2, 3
HEADER = "STRATA_WARM_PLACEMENT_V1"


def parse(text, n_layers: int, n_experts: int):
    """-> (lanes int32 [n_layers][n_experts], profile tag)."""
    raw = text.encode() if isinstance(text, str) else bytes(text)
    lanes = np.zeros((n_layers, n_experts), np.int32)
    tag = C.c_uint64(0)
    err = ErrorV1()
    check(lib.clb_placement_parse(raw, len(raw), n_layers, n_experts, C.c_void_p(lanes.ctypes.data), C.byref(tag),
                                  C.byref(err)), err)
    return lanes, int(tag.value)


def format_placement(lanes, tag: int = 0) -> str:
    lanes = np.asarray(lanes)
    nl, ne = lanes.shape
    if lanes.min() < 0 or lanes.max() > CUDA:
        raise ValueError("lane out of range")
    rows = "".join(f"{l} {e} {int(lanes[l, e])}\n" for l in range(nl) for e in range(ne))
    return f"{HEADER} {nl} {ne} {int(tag)}\n" + rows


def greedy(counts, nbytes, capacity: int, lane: int = CUDA, floor_per_layer: int = 0):
    """Place the most-selected experts per byte on `lane` until `capacity` bytes are used;
    the rest stay on the CPU lane. counts/nbytes: [layers][experts] decode-profile
    selection counts and resident bytes. floor_per_layer: experts every layer gets first
    (hottest of the layer), as crosslane keeps every layer covered on its GPU lanes.
    Deterministic: ties go to the lower (layer, expert)."""
    counts = np.asarray(counts, np.float64)
    nbytes = np.asarray(nbytes, np.int64)
    nl, ne = counts.shape
    lanes = np.zeros((nl, ne), np.int32)
    used = 0
    if floor_per_layer:
        for l in range(nl):
            order = sorted(range(ne), key=lambda e: (-counts[l, e], e))[:floor_per_layer]
            for e in order:
                if used + nbytes[l, e] <= capacity:
                    lanes[l, e] = lane
                    used += int(nbytes[l, e])
    order = sorted(((l, e) for l in range(nl) for e in range(ne)),
                   key=lambda k: (-counts[k] / max(int(nbytes[k]), 1), k))
    for l, e in order:
        if lanes[l, e] == lane:
            continue
        if used + nbytes[l, e] <= capacity:
            lanes[l, e] = lane
            used += int(nbytes[l, e])
    return lanes


def measure_cuda_costs(bank, layers=None, picks: int = 6, reps: int = 8, seed: int = 0):
    """Per-layer per-selection service ns of this lane: clb_bank_compute_many over `picks`
    resident experts of the layer (host x in, rows out), median over `reps`, divided by the
    picks. Returns {layer: ns}. Layers without `picks` resident experts are skipped."""
    rng = np.random.default_rng(seed)
    out = {}
    for layer in (range(bank.n_layers) if layers is None else layers):
        ids = [e for e in range(bank.n_experts) if bank.warm_contains(layer, e)]
        if len(ids) < picks:
            continue
        times = []
        for r in range(reps + 1):
            sel = np.sort(rng.choice(ids, picks, replace=False)).astype(np.int32)
            x = rng.standard_normal(bank.dim).astype(np.float32)
            t0 = time.perf_counter_ns()
            bank.warm_compute_many(layer, sel, x)
            if r:
                times.append(time.perf_counter_ns() - t0)
        out[layer] = float(np.median(times)) / picks
    return out


def rebalance_costs(cuda_ns, cpu_ns, decode_tokens: int, profile_bytes: bytes, gpu_slot: str = "hip",
                    other_ns=None, evidence=None):
    """A strata-warm-costs-v1 document for crosslane's optimiser (rebalance.py) with the
    CUDA lane in the `gpu_slot` column (the optimiser knows the lanes cpu/hip/sycl): per
    layer {per_expert_ns, issue_ns: 0}; cuda_ns / cpu_ns / other_ns: {layer: per-selection
    ns}. other_ns: the measured costs of the lane in the other GPU column (a B65 next to the
    CUDA lane in the HIP slot, say). Without it that column is an unused lane: the
    optimiser still requires a positive cost there, so it gets the CPU lane's (it can win
    nothing), and the plan must give that lane no room (warm_hip_room_bytes = 0 for the
    HIP column; the SYCL column carries the optimiser's per-layer coverage floor, so a lone
    CUDA lane takes gpu_slot="sycl")."""
    if gpu_slot not in ("hip", "sycl"):
        raise ValueError("gpu_slot must be one of the optimiser's GPU lanes")
    layers = sorted(set(cuda_ns) | set(cpu_ns))
    if layers != list(range(len(layers))):
        raise ValueError("costs must cover layers 0..n-1")
    rows = []
    for l in layers:
        if l not in cuda_ns or l not in cpu_ns or (other_ns is not None and l not in other_ns):
            raise ValueError(f"layer {l} lacks a measured cost")
        row = {"cpu": {"per_expert_ns": float(cpu_ns[l]), "issue_ns": 0, "measurement_source": "caller"},
               gpu_slot: {"per_expert_ns": float(cuda_ns[l]), "issue_ns": 0,
                          "measurement_source": "crosslane_b200 clb_bank_compute_many per selection"}}
        other = "sycl" if gpu_slot == "hip" else "hip"
        if other_ns is not None:
            row[other] = {"per_expert_ns": float(other_ns[l]), "issue_ns": 0, "measurement_source": "caller"}
        else:
            row[other] = {"per_expert_ns": float(cpu_ns[l]), "issue_ns": 0,
                          "measurement_source": "unused lane (no room in the plan)"}
        rows.append(row)
    return {"schema": "strata-warm-costs-v1", "scope": "measured-decode-excluding-warmup",
            "decode_tokens": int(decode_tokens), "profile_sha256": hashlib.sha256(profile_bytes).hexdigest(),
            "layers": rows, "evidence": evidence or {"lane": "cuda", "gpu_slot": gpu_slot}}
