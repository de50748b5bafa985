"""Benchmark: routed-expert decode tok/s through the 40-layer synthetic stack.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE config 3 at batch 1): 40 layers x 384 SwiGLU experts, hidden 7168,
intermediate 1536, IQ2_XXS / IQ2_XS / IQ1_M drawn per (layer, expert) from the seed
(~129.5 GB of packed weights resident in HBM), top-6 routing per layer from N(0,1)
logits (uniformly random experts), x_{l+1} = x_l + combine_l. One step = one token
through all 40 layers.

  value  : tokens/s with inputs resident in HBM, CUDA events on the bank stream (one
           routing kernel + one persistent stack kernel per token).
  e2e    : tokens/s through clb_stack_decode (host x and logits in, host routing,
           x + routes up, h down).
  roofline: the persistent stack kernel (clb::k_stack), which is the whole timed step
           apart from the routing kernel: achieved = algorithmic bytes of one token (the
           packed gate+up+down payload of every picked expert of every layer + the
           residual stream in/out) / the CUDA-event step time.
  cpu_baseline: crosslane's own CPU-lane arithmetic (q8k_core.hpp, built into
           oracle/_ref/libref.so) on a persistent 64-row-job team over all host
           threads, one token-layer sample, extrapolated to the 40-layer stack.

With --gpus N (torchrun), the ranks shard the experts by ID and decode the same token
stream together (the rows of each layer exchanged by peer stores inside the stack kernel;
scaling "strong"); --replicas runs independent full-bank replicas instead (value = the sum
over ranks of tokens / the slowest rank's time, scaling "weak").

Other workloads (own JSON line each, same keys):
  --prefill : BASELINE config 4, 2048 tokens through one 384-expert IQ2_XXS layer per step
              (grouped tcgen05 GEMMs; roofline "tensor").
  --skewed  : BASELINE config 5, a batch of 64 tokens through the 40-layer stack per step
              with Zipf(1.1) routing (clb_stack_batch; at N GPUs expert-ID sharded with an
              NCCL all-reduce of the expert rows per layer; roofline "hbm" over the distinct
              experts' bytes).
  --phase-trace : config 3 through the phase-trace build of the library (build it with
              `python crosslane_b200/build.py --trace`): per-phase durations of the stack
              kernel per token-layer from %globaltimer stamps, medians over CTAs and layers
              (one JSON line per rank; a measurement aid, not a throughput line).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIM, FF, EXPERTS, LAYERS, PICKS = 7168, 1536, 384, 40, 6
SEED, POLICY = 20261201, 2
FALLBACK_HBM_GBS = 6650.0
METRIC = "routed-expert decode tok/s (40-layer stack)"
WORKLOAD = "BASELINE config 3: 40-layer routed-expert stack, batch-1 decode"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, read through NVML every 2 ms
    by a thread while the timed region runs (read-only queries; a timed region of a few
    tens of ms still gets samples). Falls back to `nvidia-smi -lms 50` without NVML."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device, period_s=0.002):
        self.device = device
        self.period = period_s
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []  # (sm_mhz, max_mhz, reason bits)
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.device).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def __enter__(self):
        try:
            self.nvml, h = self._nvml_handle()
            pn = self.nvml
            self.bits = {"hw_slowdown": pn.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": pn.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": pn.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": pn.nvmlClocksEventReasonSwPowerCap}
            mx = pn.nvmlDeviceGetMaxClockInfo(h, pn.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    try:
                        self.samples.append((pn.nvmlDeviceGetClockInfo(h, pn.NVML_CLOCK_SM), mx,
                                             pn.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        pass
                    self.stop.wait(self.period)

            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        for s, m, r in self.samples:
            sm.append(float(s))
            mx.append(float(m))
            reasons.update(n for n, b in self.bits.items() if r & b)
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(self.NAMES, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.samples else "nvidia-smi"}


def make_inputs(rng, n, layers=LAYERS, experts=EXPERTS):
    xs = rng.standard_normal((n, DIM)).astype(np.float32)
    logits = rng.standard_normal((n, layers, experts)).astype(np.float32)
    return xs, logits


class CpuLaneTokens:
    """Whole config-3 tokens through the timed CPU expert lane (oracle/liblane.so: crosslane's
    q8k_core.hpp arithmetic vectorised with AVX2, pinned bit-identical to the reference
    compiled here; layer-batched like the reference lane's Lane::experts on a persistent
    team of all host threads). Per layer: x = RMSNorm(h), the 6 picked experts, the
    ascending-id fma combine, h += it -- the GPU step's work on the host. The weights of
    `pool` token-layers (6 config-3 experts each, ~50 MB per slot, generated once, outside
    the timed region, 0 store readers) are cycled through the 40 layers, so every layer
    streams its experts from host memory (the pool exceeds the last-level cache)."""

    def __init__(self, pool=8, threads=0, seed=99):
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import oracle_lib
        self.orc = oracle_lib.Oracle()
        self.lane = oracle_lib.cpu_lane()
        if self.lane is None:
            raise RuntimeError("oracle/liblane.so is not built")
        self.threads = threads
        rng = np.random.default_rng(seed)
        self.slots = []
        for s in range(pool):
            ids, _ = self.orc.route_sigmoid(rng.standard_normal(EXPERTS).astype(np.float32), PICKS)
            ts = [self.orc.expert_type(POLICY, SEED, s, int(e)) for e in ids]
            mats = [[self.orc.synth_matrix(t, SEED, s, int(e), r, *((FF, DIM) if r < 2 else (DIM, FF)))
                     for r in range(3)] for t, e in zip(ts, ids)]
            self.slots.append((np.asarray(ids, np.int32), ts, mats))
        self.cores = self.lane.L.lane_team_threads(threads)

    def token(self, h0, logits):
        """One token through LAYERS layers; returns (h, seconds)."""
        t0 = time.perf_counter()
        h = np.ascontiguousarray(h0, np.float32).copy()
        for l in range(LAYERS):
            ids, ts, mats = self.slots[l % len(self.slots)]
            _, w = self.orc.route_sigmoid(logits[l], PICKS)
            y, _ = self.lane.experts(ts, [m[0] for m in mats], [m[1] for m in mats], [m[2] for m in mats],
                                     self.orc.rmsnorm(h), DIM, FF, 0.0, self.threads)
            h = (h + self.orc.combine(ids, w, y)).astype(np.float32)
        return h, time.perf_counter() - t0


def cpu_baseline(tokens=3, threads=0):
    """The CPU lane timed on `tokens` whole config-3 tokens (median / min / max)."""
    try:
        run = CpuLaneTokens(threads=threads)
    except RuntimeError:
        return None
    rng = np.random.default_rng(7)
    run.token(rng.standard_normal(DIM).astype(np.float32), rng.standard_normal((LAYERS, EXPERTS)).astype(np.float32))
    times = [run.token(rng.standard_normal(DIM).astype(np.float32),
                       rng.standard_normal((LAYERS, EXPERTS)).astype(np.float32))[1] for _ in range(tokens)]
    med = statistics.median(times)
    return {"value": 1.0 / med, "unit": "tok/s", "cores": int(run.cores), "kind": "port",
            "sample": f"{tokens} whole config-3 tokens (40 layers x 6 experts, mixed IQ2_XXS/IQ2_XS/IQ1_M) after one "
                      f"warm-up token; {med * 1e3:.1f} ms per token median, {min(times) * 1e3:.1f} min, "
                      f"{max(times) * 1e3:.1f} max; crosslane's q8k_core.hpp arithmetic vectorised with AVX2 "
                      f"(bit-identical to it), layer-batched like Lane::experts on {run.cores} host threads; "
                      f"weights generated in host memory (0 store readers)",
            "repeats": {"runs": tokens, "median_ms": round(med * 1e3, 2), "min_ms": round(min(times) * 1e3, 2),
                        "max_ms": round(max(times) * 1e3, 2)}}


def config3(args, world, sharded):
    return {"workload": WORKLOAD, "layers": args.layers, "experts": args.experts, "dim": DIM, "ff": FF, "picks": PICKS,
            "types": "IQ2_XXS/IQ2_XS/IQ1_M per (layer, expert), seed-drawn", "batch": 1,
            "routing": "top-6 by sigmoid of N(0,1) logits, renormalised",
            "parallelism": (f"expert-ID sharded x{world} (peer-store row exchange in the stack kernel)"
                            if sharded else f"replica x{world}" if world > 1 else "single GPU"),
            "summation": "exact reference order" if args.exact_order
            else "segmented rows, fixed-order partials (run-to-run identical)",
            "l2": "inputs larger than L2: each token streams ~2 GB of distinct expert weights"}


def _all_same(vals, world):
    """True when every rank holds the same bytes (an all-gather of a digest over the process
    group); vals: this rank's array."""
    import hashlib
    import torch.distributed as dist
    digest = hashlib.sha256(np.ascontiguousarray(vals).tobytes()).hexdigest()
    if world == 1:
        return True
    out = [None] * world
    dist.all_gather_object(out, digest)
    return all(d == out[0] for d in out)


def parity_config3(args, rank, world, sharded, bank, local):
    """Correctness of the benchmarked configuration, checked after the timed region on every
    rank: (1) a 3-layer exact-order bank of the same weights (expert-ID sharded like the
    benchmarked one) decodes 2 tokens back to back; the residual stream is identical on every
    rank and equal bit for bit to the CPU oracle's stack (crosslane's q8k_core.hpp arithmetic
    and the ascending-id fma combine, runtime.cpp:184-187); (2) the benchmarked fast-order
    bank's first layer, fed the same input, is within the north-star tolerance of the
    oracle's layer (relative L2 <= 1e-3, max-abs-relative <= 5e-3); (3) a whole 40-layer
    fast-order token is identical on every rank."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib
    import crosslane_b200 as cb
    orc = oracle_lib.Oracle()
    rng = np.random.default_rng(4040)  # the same inputs on every rank
    n_ex = 3
    x0 = rng.standard_normal(DIM).astype(np.float32)
    logits = rng.standard_normal((2, args.layers, args.experts)).astype(np.float32)
    if sharded:
        from crosslane_b200.sharded import ShardedBank
        ex = ShardedBank(n_layers=n_ex, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local,
                         rank=rank, world=world, exact_order=True)
    else:
        ex = cb.ExpertBank(n_layers=n_ex, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local,
                           exact_order=True)
    try:
        ex.fill_synthetic(SEED, args.policy)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        outs, h = [], x0
        for t in range(2):
            h = ex.stack_decode(0, n_ex, h, logits[t, :n_ex])
            outs.append(h)
    finally:
        ex.close()
    # fast order (the benchmarked bank): one layer against the oracle, a whole token across
    # ranks. Every sharded decode runs before the host oracle below, so that no rank waits in
    # a kernel for a peer that is still busy on the host.
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    one = bank.stack_decode(0, 1, x0, logits[0, :1])
    full = bank.stack_decode(0, args.layers, x0, logits[0])
    exact_same = _all_same(np.stack(outs), world)
    fast_same = _all_same(np.stack([one, full]), world)
    exact_bits = None
    if rank == 0:
        want, exact_bits = x0, True
        for t in range(2):
            want = orc.stack(args.policy, SEED, want, logits[t, :n_ex], DIM, FF, k=PICKS)
            exact_bits = exact_bits and bool(np.array_equal(oracle_lib.bits(outs[t]), oracle_lib.bits(want)))
    rl2 = mar = None
    if rank == 0:
        want1 = orc.stack(args.policy, SEED, x0, logits[0, :1], DIM, FF, k=PICKS)
        rl2, mar = oracle_lib.rel_l2(one, want1), oracle_lib.max_abs_rel(one, want1)
    ok = None
    if rank == 0:
        ok = bool(exact_same and exact_bits and fast_same and rl2 <= 1e-3 and mar <= 5e-3)
    return {"ok": ok, "ranks": world, "exact_order_layers": n_ex, "exact_order_tokens": 2,
            "exact_ranks_identical": exact_same, "exact_bitexact_vs_oracle": exact_bits,
            "fast_layer_rel_l2": rl2, "fast_layer_max_abs_rel": mar, "fast_tolerance": [1e-3, 5e-3],
            "fast_40_layer_token_ranks_identical": fast_same}


def run_reference(args, rank, world):
    """The reference arm: the CPU lane on `steps` whole tokens (each step is timed and is
    one token through the 40-layer stack), after `warmup` untimed tokens."""
    if rank != 0:
        return
    try:
        run = CpuLaneTokens()
    except RuntimeError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"CPU lane not built: {e}"}))
        return
    rng = np.random.default_rng(7)
    for _ in range(args.warmup):
        run.token(rng.standard_normal(DIM).astype(np.float32), rng.standard_normal((LAYERS, EXPERTS)).astype(np.float32))
    times = [run.token(rng.standard_normal(DIM).astype(np.float32),
                       rng.standard_normal((LAYERS, EXPERTS)).astype(np.float32))[1] for _ in range(args.steps)]
    total = sum(times)
    value = args.steps / total
    med = statistics.median(times)
    cpu = {"value": value, "unit": "tok/s", "cores": int(run.cores), "kind": "port",
           "sample": f"{args.steps} whole config-3 tokens timed, each through 40 layers (after {args.warmup} warm-up "
                     f"tokens); {med * 1e3:.1f} ms per token median; crosslane's q8k_core.hpp arithmetic vectorised "
                     f"with AVX2 (bit-identical to it), layer-batched like Lane::experts on {run.cores} host threads"}
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 and not args.replicas else "weak", "vs_baseline": None,
            "dtype": "int8xIQ/fp32", "data": "synthetic", "config": config3(args, world, world > 1 and not args.replicas),
            "impl": "reference", "cpu_baseline": cpu,
            "repeats": {"runs": args.steps, "unit": "ms per token", "median": round(med * 1e3, 2),
                        "min": round(min(times) * 1e3, 2), "max": round(max(times) * 1e3, 2)},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PF_TOKENS = 2048
PF_METRIC = "routed-expert prefill tok/s (one layer, 2048 tokens)"
PF_WORKLOAD = "BASELINE config 4: batched prefill through one MoE layer, 2048 tokens, 384 IQ2_XXS experts, top-6"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    return 1590.0, "fallback 1590 TFLOP/s"


def prefill_cpu_baseline(tokens=2, threads=0):
    """Reference CPU lane on `tokens` tokens of the config-4 layer (one token = 6 experts + combine)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib
    ref = oracle_lib.reference()
    if ref is None:
        return None
    orc = oracle_lib.Oracle()
    rng = np.random.default_rng(98)
    times, cores = [], None
    for s in range(tokens + 1):  # first token warms the team and page cache
        ids, w = orc.route_sigmoid(rng.standard_normal(EXPERTS).astype(np.float32), PICKS)
        x = rng.standard_normal(DIM).astype(np.float32)
        mats = [(orc.synth_matrix(16, SEED, 0, int(e), 0, FF, DIM), orc.synth_matrix(16, SEED, 0, int(e), 1, FF, DIM),
                 orc.synth_matrix(16, SEED, 0, int(e), 2, DIM, FF)) for e in ids]
        t0 = time.perf_counter()
        rows = np.stack([ref.expert(16, g, u, d, x, DIM, FF, 0.0, threads)[1] for g, u, d in mats])
        ref.combine(ids, w, rows)
        if s > 0:
            times.append(time.perf_counter() - t0)
        cores = ref.L.ref_team_threads(threads)
    per_tok = statistics.median(times)
    return {"value": 1.0 / per_tok, "unit": "tok/s", "cores": int(cores), "kind": "reference",
            "sample": f"{tokens} token(s) of config 4 (6 IQ2_XXS experts each, weights generated in RAM), median "
                      f"{per_tok * 1e3:.1f} ms per token; crosslane q8k_core.hpp arithmetic, persistent 64-row-job "
                      f"team (the CPU lane has no batched path: tokens run one after another)"}


def run_prefill(args, rank, world, local):
    """Config 4: T tokens through one IQ2_XXS layer per step; N>1 runs independent replicas."""
    import torch
    import torch.distributed as dist

    import crosslane_b200 as cb

    if args.impl == "reference":
        if rank != 0:
            return
        res = prefill_cpu_baseline(tokens=max(1, min(args.steps, 4)))
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref.so was not built"}))
            return
        print(json.dumps({"metric": PF_METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": PF_TOKENS * 1e3 / res["value"],
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xIQ/fp32",
                          "data": "synthetic", "config": {"workload": PF_WORKLOAD, "tokens": PF_TOKENS},
                          "impl": "reference", "cpu_baseline": res,
                          "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    T, k = PF_TOKENS, PICKS
    bank = cb.ExpertBank(n_layers=1, n_experts=args.experts, dim=DIM, ff=FF, max_picks=k, device=local)
    bank.fill_synthetic(SEED, 0)
    stream = torch.cuda.ExternalStream(bank.stream)
    rng = np.random.default_rng(2000 + rank)
    n_in = 4  # distinct batches cycled through the steps
    xs = rng.standard_normal((n_in, T, DIM)).astype(np.float32)
    ids = np.zeros((n_in, T, k), np.int32)
    ws = np.zeros((n_in, T, k), np.float32)
    for i in range(n_in):
        lg = rng.standard_normal((T, args.experts)).astype(np.float32)
        for t in range(T):
            ids[i, t], ws[i, t] = cb.route_host(0, lg[t], k)
    d_x = torch.from_numpy(xs).cuda()
    d_ids = torch.from_numpy(ids).cuda()
    d_w = torch.from_numpy(ws).cuda()
    d_out = torch.empty((T, DIM), dtype=torch.float32, device="cuda")
    d_ws = torch.empty(bank.prefill_workspace_bytes(T, k), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()

    def step(i):
        j = i % n_in
        bank.prefill_layer_device(0, d_ids[j], d_w[j], d_x[j], d_out, d_ws)

    for i in range(args.warmup):
        step(i)
    bank.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    bank.synchronize()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * T * args.steps / (ms / 1e3)
    # GEMM kernels alone (gate/up and down), for the tensor-pipe figure
    gemm_ms = 0.0
    for mask in (2, 8):
        ev0.record(stream)
        for _ in range(5):
            bank.prefill_phases_device(0, d_ids[0], d_w[0], d_x[0], d_out, d_ws, mask)
        ev1.record(stream)
        ev1.synchronize()
        gemm_ms += ev0.elapsed_time(ev1) / 5
    # e2e: host buffers through clb_prefill_layer (copies in the timed region)
    e2e_steps = 2 if args.quick else max(3, min(args.steps, 10))
    bank.prefill_layer(0, ids[0], ws[0], xs[0])
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        bank.prefill_layer(0, ids[i % n_in], ws[i % n_in], xs[i % n_in])
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    flops = 2.0 * T * k * 3 * DIM * FF  # 811.7 GFLOP per step
    peak_tf, peak_kind = tensor_peak()
    hbm, hbm_kind = peaks()
    tflops = flops / (gemm_ms / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        cpu = prefill_cpu_baseline(tokens=2)
    line = {
        "metric": PF_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 integers x fp16 integers -> fp32 (IQ2_XXS x Q8_K)", "data": "synthetic",
        "config": {"workload": PF_WORKLOAD, "tokens": T, "experts": args.experts, "dim": DIM, "ff": FF, "picks": k,
                   "routing": "top-6 by sigmoid of N(0,1) logits, renormalised",
                   "parallelism": f"replica x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: 3.27 GB of expert weights per step"},
        "e2e": {"value": round(world * T / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": T * DIM * 4 + T * k * 8,
                "d2h_bytes_per_step": T * DIM * 4},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": round(tflops / peak_tf, 4), "traffic": None, "kernel": "clb::k_prefill_gemm (both roles)",
                     "peak_source": peak_kind, "algorithmic_flops_per_step": flops,
                     "gemm_ms_per_step": round(gemm_ms, 4),
                     "hbm_frac_of_step": round(bank.weight_bytes / (ms_per_step / 1e3) / 1e9 / hbm, 4),
                     "hbm_peak_source": hbm_kind},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": 7 * args.steps,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    bank.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


SK_BATCH = 64
SK_METRIC = "routed-expert decode tok/s (40-layer stack, batch 64, Zipf(1.1) routing)"
SK_WORKLOAD = "BASELINE config 5: skewed-routing decode at batch 64 through the 40-layer stack"


def zipf_logits(rng, layers, T, E, s=1.1):
    """[layers][T][E] router logits whose top-k follows Zipf(s) expert popularity over a
    per-layer seeded permutation of the experts: log p(rank) + Gumbel noise per token, so
    top-k of the logits is a draw of k distinct experts with probabilities p (Gumbel top-k)."""
    logp = -s * np.log(np.arange(1, E + 1, dtype=np.float64))
    out = np.empty((layers, T, E), np.float32)
    for l in range(layers):
        rank = np.argsort(np.random.default_rng(SEED + 7919 * l).permutation(E))  # rank of expert e
        out[l] = (logp[rank][None, :] + rng.gumbel(size=(T, E))).astype(np.float32)
    return out


def shard_load(ids_by_layer, experts, world):
    """Mean over layers of (max over GPUs / mean over GPUs) of the distinct picked experts each
    GPU decodes (its share of the layer's weight reads) when experts are split into `world`
    contiguous ID blocks; ids_by_layer: [layers][tokens][k]."""
    ratios = []
    for ids in ids_by_layer:
        owner = np.minimum((np.unique(np.asarray(ids)) * world) // experts, world - 1)
        load = np.bincount(owner, minlength=world)
        ratios.append(load.max() / load.mean())
    return float(np.mean(ratios))


def run_skewed(args, rank, world, local):
    """Config 5: a batch of 64 tokens (one per sequence) through the 40-layer stack per step,
    Zipf(1.1) routing, each layer one grouped prefill over the batch (clb_stack_batch)."""
    import torch

    import crosslane_b200 as cb

    if args.impl == "reference":
        if rank != 0:
            return
        res = cpu_baseline(tokens=3)
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref.so was not built"}))
            return
        print(json.dumps({"metric": SK_METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": SK_BATCH * 1e3 / res["value"], "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "int8xIQ/fp32", "data": "synthetic",
                          "config": {"workload": SK_WORKLOAD, "batch": SK_BATCH}, "impl": "reference",
                          "cpu_baseline": res,
                          "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    T, k, L = SK_BATCH, PICKS, args.layers
    if world > 1:  # expert-ID sharding: rank r holds experts [r*E/N, (r+1)*E/N); rows summed over NCCL per layer
        from crosslane_b200.sharded import ShardedBank
        bank = ShardedBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=k, device=local, rank=rank,
                           world=world)
    else:
        bank = cb.ExpertBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=k, device=local)
    bank.fill_synthetic(SEED, args.policy)
    stream = torch.cuda.ExternalStream(bank.stream)
    rng = np.random.default_rng(5000)  # the same batch on every rank
    n_in = 3
    xs = rng.standard_normal((n_in, T, DIM)).astype(np.float32)
    lgs = np.stack([zipf_logits(rng, L, T, args.experts) for _ in range(n_in)])
    # algorithmic bytes: every distinct picked expert of every layer read once (summed over the
    # ranks that own them), + h in/out per layer
    own_b, own_e = (bank.expert_begin, bank.expert_end) if world > 1 else (0, args.experts)
    alg, distinct = [], []
    for i in range(n_in):
        tot = 0
        for l in range(L):
            picked = set()
            for t in range(T):
                ids, _ = cb.route_host(0, lgs[i, l, t], k)
                picked.update(int(e) for e in ids)
            tot += sum(bank.expert_info(l, e)[1] for e in picked if own_b <= e < own_e)
            distinct.append(len(picked))
        alg.append(tot)
    if world > 1:
        t = torch.tensor(alg, dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        alg = t.cpu().tolist()
    alg_bytes = float(np.mean(alg)) + L * 2 * T * DIM * 4
    routes0 = [[cb.route_host(0, lgs[0, l, t], k)[0] for t in range(T)] for l in range(L)]
    d_x = torch.from_numpy(xs).cuda()
    d_lg = torch.from_numpy(lgs).cuda()
    d_h = torch.empty((T, DIM), dtype=torch.float32, device="cuda")
    d_ws = torch.empty(bank.stack_batch_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    d_rows = torch.zeros((T * k, DIM), dtype=torch.float32, device="cuda") if world > 1 else None
    torch.cuda.synchronize()

    def run(j):
        if world > 1:
            bank.stack_batch_device(0, L, d_h, d_lg[j], d_ws, d_rows)
        else:
            bank.stack_batch_device(0, L, d_h, d_lg[j], d_ws)

    def step(i):
        j = i % n_in
        with torch.cuda.stream(stream):
            d_h.copy_(d_x[j])
        run(j)

    for i in range(args.warmup):
        step(i)
    bank.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    bank.synchronize()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)
    # e2e: host h and logits in, h out, through the public API
    e2e_steps = 2 if args.quick else max(2, min(args.steps, 5))
    if world == 1:  # clb_stack_batch: host routing, copies inside the call
        bank.stack_batch(0, L, xs[0], lgs[0])
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            bank.stack_batch(0, L, xs[i % n_in], lgs[i % n_in])
        e2e_s = (time.perf_counter() - t0) / e2e_steps
    else:  # pinned host buffers up, the sharded device path, h down
        hx = torch.from_numpy(xs).pin_memory()
        hl = torch.from_numpy(lgs).pin_memory()
        hout = torch.empty((T, DIM), dtype=torch.float32).pin_memory()
        d_l1 = torch.empty_like(d_lg[0])

        def e2e_step(i):
            j = i % n_in
            with torch.cuda.stream(stream):
                d_h.copy_(hx[j], non_blocking=True)
                d_l1.copy_(hl[j], non_blocking=True)
            bank.stack_batch_device(0, L, d_h, d_l1, d_ws, d_rows)
            with torch.cuda.stream(stream):
                hout.copy_(d_h, non_blocking=True)
            stream.synchronize()

        e2e_step(0)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            e2e_step(i)
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    hbm, hbm_kind = peaks()
    achieved = alg_bytes / (ms_per_step / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        cpu = cpu_baseline(tokens=3)
        if cpu is not None:
            cpu["sample"] += "; the CPU lane decodes the batch token by token (no batched path)"
    line = {
        "metric": SK_METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "fp16 integers x fp16 integers -> fp32 (IQ x Q8_K)", "data": "synthetic",
        "config": {"workload": SK_WORKLOAD, "batch": T, "layers": L, "experts": args.experts, "dim": DIM, "ff": FF,
                   "picks": k, "types": "IQ2_XXS/IQ2_XS/IQ1_M per (layer, expert)",
                   "routing": "top-6 of log Zipf(1.1) over a per-layer seeded permutation + Gumbel noise",
                   "distinct_experts_per_layer": round(float(np.mean(distinct)), 1),
                   "shard_load_max_over_mean": round(shard_load(routes0, args.experts, world), 3),
                   "parallelism": f"expert-ID sharded x{world}, rows all-reduced over NCCL per layer" if world > 1
                   else "single GPU",
                   "l2": "inputs larger than L2: %.1f GB of distinct expert weights per step" % (alg_bytes / 1e9)},
        "e2e": {"value": round(T / e2e_s, 1), "unit": "tok/s",
                "h2d_bytes_per_step": T * DIM * 4 + L * T * k * 8, "d2h_bytes_per_step": T * DIM * 4},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm * world, "unit": "GB/s",
                     "frac": round(achieved / (hbm * world), 4), "traffic": None,
                     "kernel": "whole step (per layer: route, group, norm+Q8_K, gather, 2 x clb::k_prefill_gemm, "
                               "SwiGLU+Q8_K, combine)",
                     "algorithmic_bytes_per_step": alg_bytes, "peak_source": hbm_kind},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": 11 * L * args.steps,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    # tensors used on the bank stream (the all-reduce recorded it on them) go before the stream
    torch.cuda.synchronize()
    del d_x, d_lg, d_h, d_ws, d_rows
    if world > 1:
        del hx, hl, hout, d_l1
    torch.cuda.synchronize()
    bank.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


PHASES = ["h", "norm", "gateup", "gateup_end", "qh_wait", "down", "combine_barrier"]


def run_phase_trace(args, rank, world, local):
    """Config 3 through the phase-trace build: `steps` tokens after `warmup`, and for each
    phase boundary of the stack kernel the duration per token-layer (median over CTAs and
    over layers 1..L-1; layer 0 also stages the tables), plus the slowest CTA's (mean over
    layers) and, sharded, a split by the number of picks this GPU owned in the layer."""
    import ctypes as C
    lib_path = os.path.join(ROOT, "crosslane_b200", "libcrosslane_b200_trace.so")
    if not os.path.exists(lib_path):
        raise SystemExit("phase trace: build it first with `python crosslane_b200/build.py --trace`")
    os.environ["CROSSLANE_B200_LIB"] = lib_path
    import torch
    import torch.distributed as dist

    import crosslane_b200 as cb
    from crosslane_b200._capi import lib

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    L = args.layers
    if world > 1:
        from crosslane_b200.sharded import ShardedBank
        bank = ShardedBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local,
                           rank=rank, world=world, exact_order=args.exact_order)
    else:
        bank = cb.ExpertBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local,
                             exact_order=args.exact_order)
    bank.fill_synthetic(SEED, args.policy)
    if world > 1:
        dist.barrier()
    stream = torch.cuda.ExternalStream(bank.stream)
    rng = np.random.default_rng(1000)  # the same tokens on every rank
    n_layers, n_ctas, n_slots = 64, 160, 8  # the kernel's trace array
    lib.clb_stack_trace_read.restype = C.c_int
    lib.clb_stack_trace_read.argtypes = [C.c_void_p, C.c_size_t]
    grid = torch.cuda.get_device_properties(local).multi_processor_count
    per, kowns, ms_all = [], [], []
    for i in range(args.warmup + args.steps):
        x = torch.from_numpy(rng.standard_normal(DIM).astype(np.float32)).cuda()
        lg = rng.standard_normal((L, args.experts)).astype(np.float32)
        d_lg = torch.from_numpy(lg).cuda()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        bank.stack_decode_device(0, L, x, d_lg)
        ev1.record(stream)
        ev1.synchronize()
        if i < args.warmup:
            continue
        buf = np.zeros(n_layers * n_ctas * n_slots, np.uint64)
        if lib.clb_stack_trace_read(buf.ctypes.data, buf.nbytes) != 0:
            raise SystemExit("phase trace: clb_stack_trace_read failed")
        t = buf.reshape(n_layers, n_ctas, n_slots)[:L, :grid].astype(np.int64)
        per.append(np.diff(t, axis=2)[1:] / 1e3)  # [layer][cta][phase] us
        kowns.append([sum(1 for e in cb.route_host(0, lg[l], PICKS)[0] if bank.expert_begin <= int(e) < bank.expert_end)
                      for l in range(1, L)])
        ms_all.append(ev0.elapsed_time(ev1))
    d = np.concatenate(per)  # [tokens * (L - 1)][cta][phase]
    k_all = np.concatenate(kowns)
    phases = {name: {"median_us": round(float(np.median(d[:, :, j])), 2),
                     "slowest_cta_us": round(float(np.mean(d[:, :, j].max(axis=1))), 2)}
              for j, name in enumerate(PHASES) if name != "gateup_end"}
    span = [float(np.median(p.sum(axis=2))) for p in per]  # per token: median CTA's layer time
    line = {"metric": "stack kernel phase trace", "rank": rank, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "us_per_token_layer": round(float(np.mean(ms_all)) * 1e3 / L, 2),
            "token_ms": round(float(np.mean(ms_all)), 4), "phases": phases,
            "layer_span_median_us": round(float(np.mean(span)), 2),
            "config": config3(args, world, world > 1), "library": "libcrosslane_b200_trace.so (-DCLB_FLOW_TRACE)"}
    if world > 1:
        by = {}
        for kk in sorted(set(int(v) for v in k_all)):
            idx = k_all == kk
            by[str(kk)] = {"layers": int(idx.sum()), **{name: round(float(np.median(d[idx][:, :, j])), 2)
                                                       for j, name in enumerate(PHASES) if name != "gateup_end"}}
        line["by_owned_picks"] = by
    print(json.dumps(line), flush=True)
    bank.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS, help="smaller stacks for quick checks only")
    ap.add_argument("--experts", type=int, default=EXPERTS,
                    help="experts per layer (profiling captures only: a small bank, same per-token work)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the correctness check after the timed region")
    ap.add_argument("--policy", type=int, default=POLICY, help="quant type policy of the bank (2 = config 3 mix)")
    ap.add_argument("--quick", action="store_true", help="skip the e2e pass and the CPU baseline (tuning sweeps)")
    ap.add_argument("--replicas", action="store_true",
                    help="with N>1: independent full-bank replicas per GPU instead of expert-ID sharding")
    ap.add_argument("--exact-order", action="store_true",
                    help="reference summation order (CLB_BANK_EXACT_ORDER): bit-identical to the CPU lane")
    ap.add_argument("--skewed", action="store_true",
                    help="BASELINE config 5: batch-64 decode through the stack with Zipf(1.1) routing")
    ap.add_argument("--prefill", action="store_true",
                    help="BASELINE config 4 instead: 2048 tokens through one IQ2_XXS layer per step (own JSON line)")
    ap.add_argument("--phase-trace", action="store_true",
                    help="per-phase durations of the stack kernel (the -DCLB_FLOW_TRACE build of the library)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.prefill:
        if args.steps == 200:
            args.steps = 20
        return run_prefill(args, rank, world, local)
    if args.skewed:
        if args.steps == 200:
            args.steps = 10
        return run_skewed(args, rank, world, local)
    if args.phase_trace:
        if args.steps == 200:
            args.steps = 4
        return run_phase_trace(args, rank, world, local)

    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist

    import crosslane_b200 as cb

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    L = args.layers
    sharded = world > 1 and not args.replicas
    if sharded:  # expert-ID sharding: rank r holds experts [r*E/N, (r+1)*E/N), rows exchanged over NVLink
        from crosslane_b200.sharded import ShardedBank
        bank = ShardedBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local, rank=rank,
                           world=world, exact_order=args.exact_order)
    else:
        bank = cb.ExpertBank(n_layers=L, n_experts=args.experts, dim=DIM, ff=FF, max_picks=PICKS, device=local,
                             exact_order=args.exact_order)
    t0 = time.time()
    bank.fill_synthetic(SEED, args.policy)
    fill_s = time.time() - t0
    if world > 1:
        dist.barrier()  # every bank filled before the first (exchanging) launch
    stream = torch.cuda.ExternalStream(bank.stream)

    rng = np.random.default_rng(1000 if sharded else 1000 + rank)  # sharded: every rank decodes the same tokens
    n_in = args.warmup + args.steps
    xs, logits = make_inputs(rng, n_in, L, args.experts)
    d_xs = torch.from_numpy(xs).cuda()
    d_logits_all = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    d_x = torch.empty(DIM, dtype=torch.float32, device="cuda")
    d_lg = torch.empty((L, args.experts), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step(i):
        with torch.cuda.stream(stream):
            d_x.copy_(d_xs[i], non_blocking=True)
            d_lg.copy_(d_logits_all[i], non_blocking=True)
        bank.stack_decode_device(0, L, d_x, d_lg)

    for i in range(args.warmup):
        step(i)
    bank.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # the K timed steps, with events also at the thirds: three repetitions of K/3 steps
    # (median / min / max) inside the one timed region
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    cuts = [0, args.steps // 3, 2 * args.steps // 3, args.steps]
    with ClockSampler(local) as clocks:
        evs[0].record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
            for c in (1, 2):
                if i + 1 == cuts[c]:
                    evs[c].record(stream)
        evs[3].record(stream)
        evs[3].synchronize()
    torch.cuda.synchronize()
    ms = evs[0].elapsed_time(evs[3])
    reps = [evs[c].elapsed_time(evs[c + 1]) / (cuts[c + 1] - cuts[c]) for c in range(3) if cuts[c + 1] > cuts[c]]
    if world > 1:
        t = torch.tensor([ms] + reps, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, reps = float(t[0].item()), [float(v) for v in t[1:].tolist()]
        dist.barrier()
    ms_per_step = ms / args.steps
    units_r = 1 if (world > 1 and not args.replicas) else world
    repeats = {"runs": len(reps), "unit": "tok/s",
               "median": round(units_r * 1e3 / statistics.median(reps), 2) if reps else None,
               "min": round(units_r * 1e3 / max(reps), 2) if reps else None,
               "max": round(units_r * 1e3 / min(reps), 2) if reps else None}
    units = 1 if sharded else world  # tokens per step of the whole job
    value = units * args.steps / (ms / 1e3)

    # ---- e2e through the host-buffer C ABI call (copies inside the timed region) ----
    hx = np.ascontiguousarray(xs)
    hl = np.ascontiguousarray(logits)
    e2e_steps = 1 if args.quick else args.steps
    for i in range(0 if args.quick else args.warmup):
        bank.stack_decode(0, L, hx[i], hl[i])
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        bank.stack_decode(0, L, hx[args.warmup + i], hl[args.warmup + i])
    e2e_s = time.perf_counter() - t0
    e2e_s = e2e_s * args.steps / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = {"value": units * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * DIM + 8 * L * PICKS,
           "d2h_bytes_per_step": 4 * DIM}

    # ---- roofline: algorithmic bytes of one token through the stack kernel ----
    peak, peak_kind = peaks()
    step_bytes = []
    own_b, own_e = bank.expert_begin, bank.expert_end
    for i in range(args.steps):
        tok = args.warmup + i
        nbytes = 0 if (sharded and rank != 0) else 8 * DIM  # residual stream in and out, once per token
        for layer in range(L):
            ids, _ = cb.route_host(0, logits[tok, layer], PICKS)
            nbytes += sum(bank.expert_info(layer, int(e))[1] for e in ids if own_b <= int(e) < own_e)
        step_bytes.append(nbytes)
    bytes_per_step = float(np.mean(step_bytes))  # this rank's share
    if world > 1:
        t = torch.tensor([bytes_per_step], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)  # whole job: every rank's share (replicas: every rank's own token)
        bytes_per_step = float(t.item())
    peak_job = peak * world  # each GPU streams its own HBM
    step_gbs = bytes_per_step / (ms_per_step / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "k_stack_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            t = json.load(f)
        # measured DRAM bytes per token-layer on a small capture, scaled to this stack
        traffic = round(t["dram_bytes_per_token_layer"] * L) if "dram_bytes_per_token_layer" in t else None
    roofline = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak_job, "unit": "GB/s",
                "frac": round(step_gbs / peak_job, 4), "traffic": traffic, "kernel": "clb::k_stack",
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "algorithmic_bytes_per_launch": int(bytes_per_step),
                "avg_launch_us": round(ms_per_step * 1e3, 2),
                "launch_timing": "CUDA events around each step's routing + stack launches"}

    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        cpu = cpu_baseline(tokens=max(3, min(args.steps, 20)))
    parity = None if args.no_parity else parity_config3(args, rank, world, sharded, bank, local)

    clk = clocks.summary()
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": "int8xIQ/fp32", "data": "synthetic",
        "config": config3(args, world, sharded),
        "bank": {"gb": round(bank.weight_bytes / 1e9, 2), "fill_s": round(fill_s, 1)},
        "e2e": {k: (round(v, 2) if isinstance(v, float) else v) for k, v in e2e.items()},
        "repeats": repeats,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "parity": parity,
        "clocks": clk,
        "gpu_launches": 2 * args.steps if bank.persistent else (1 + 3 * L) * args.steps,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    bank.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
