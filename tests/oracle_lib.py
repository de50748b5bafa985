"""Test-side ctypes loader of the CPU oracle (oracle/liboracle.so) and of the reference
arithmetic pin (oracle/_ref/libref.so). Test infrastructure only."""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libref.so")

BLOCK_BYTES = {16: 66, 17: 74, 29: 56}
Q8K = 292
VP = C.c_void_p


def ptr(a):
    return a.ctypes.data_as(VP)


def _build_oracle():
    if not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-C", ORACLE_DIR, "liboracle.so"], check=True, capture_output=True)


class Oracle:
    def __init__(self):
        _build_oracle()
        L = C.CDLL(ORACLE_SO)
        self.L = L
        L.orc_half.restype = C.c_float
        L.orc_half.argtypes = [C.c_uint16]
        L.orc_nearest.argtypes = [C.c_float]
        L.orc_dot.restype = C.c_float
        L.orc_dot.argtypes = [C.c_int, VP, VP, C.c_int]
        L.orc_swiglu.restype = C.c_float
        L.orc_swiglu.argtypes = [C.c_float, C.c_float, C.c_float]
        L.orc_block_scale.restype = C.c_float
        L.orc_block_scale.argtypes = [C.c_int, VP]
        L.orc_synth_matrix.argtypes = [C.c_int, C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.c_int,
                                       VP, VP]
        L.orc_expert_type.argtypes = [C.c_int, C.c_uint64, C.c_uint32, C.c_uint32]
        L.orc_layer_synth.argtypes = [C.c_int, C.c_uint64, C.c_uint32, VP, VP, C.c_int, VP, VP, C.c_int, C.c_int,
                                      C.c_float, VP, C.c_int, VP]
        L.orc_expert.argtypes = [C.c_int, VP, C.c_int, VP, C.c_int, VP, VP, C.c_int, C.c_int, C.c_float, VP, VP]
        L.orc_mv.argtypes = [C.c_int, VP, VP, VP, C.c_int, C.c_int]
        L.orc_combine.argtypes = [VP, VP, C.c_int, VP, VP, C.c_int, VP]
        L.orc_route_sigmoid.argtypes = [VP, C.c_int, C.c_int, VP, VP]
        L.orc_route_sqrt_softplus.argtypes = [VP, VP, C.c_int, C.c_int, C.c_float, VP, VP]
        L.orc_decode_sub.argtypes = [C.c_int, VP, C.c_int, VP, C.POINTER(C.c_float), VP]
        L.orc_integer_lane.argtypes = [C.c_int, VP, VP, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        self._table = None

    # ---- synthetic inputs ----
    def scale_table(self):
        if self._table is None:
            t = np.zeros(65536, np.uint16)
            self.L.orc_scale_table(ptr(t))
            self._table = t
        return self._table

    def expert_type(self, policy, seed, layer, expert):
        return self.L.orc_expert_type(policy, seed, layer, expert)

    def synth_matrix(self, qtype, seed, layer, expert, role, n, k):
        out = np.zeros(n * (k // 256) * BLOCK_BYTES[qtype], np.uint8)
        self.L.orc_synth_matrix(qtype, seed, layer, expert, role, n, k, ptr(self.scale_table()), ptr(out))
        return out

    # ---- arithmetic ----
    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * Q8K, np.uint8)
        for b in range(x.size // 256):
            self.L.orc_quant_block(ptr(x[256 * b:]), ptr(out[Q8K * b:]))
        return out

    def mv(self, qtype, w, q, n, k):
        y = np.zeros(n, np.float32)
        self.L.orc_mv(qtype, ptr(w), ptr(q), ptr(y), n, k)
        return y

    def dot(self, qtype, w_row, q, nb):
        return self.L.orc_dot(qtype, ptr(w_row), ptr(q), nb)

    def swiglu(self, g, u, limit=0.0):
        return np.array([self.L.orc_swiglu(float(a), float(b), limit) for a, b in zip(g, u)], np.float32)

    def expert(self, qtype, gate, up, down, x, dim, ff, limit=0.0):
        """qtype: one type for the three matrices, or a (gate, up, down) tuple of types."""
        tg, tu, td = qtype if isinstance(qtype, tuple) else (qtype, qtype, qtype)
        h = np.zeros(ff, np.float32)
        y = np.zeros(dim, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.L.orc_expert(tg, ptr(gate), tu, ptr(up), td, ptr(down), ptr(x), dim, ff, limit, ptr(h),
                               ptr(y))
        assert rc == 0
        return h, y

    def combine(self, ids, w, rows, shared=None):
        ids = np.ascontiguousarray(ids, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        rows = np.ascontiguousarray(rows, np.float32)
        dim = rows.shape[1]
        out = np.zeros(dim, np.float32)
        sh = np.ascontiguousarray(shared, np.float32) if shared is not None else None
        self.L.orc_combine(ptr(ids), ptr(w), len(ids), ptr(rows), ptr(sh) if sh is not None else None, dim, ptr(out))
        return out

    def route_sigmoid(self, logits, k):
        logits = np.ascontiguousarray(logits, np.float32)
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        assert self.L.orc_route_sigmoid(ptr(logits), logits.size, k, ptr(ids), ptr(w)) == 0
        return ids, w

    def route_sqrt_softplus(self, logits, bias, k, scale):
        logits = np.ascontiguousarray(logits, np.float32)
        bias = np.ascontiguousarray(bias, np.float32)
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        assert self.L.orc_route_sqrt_softplus(ptr(logits), ptr(bias), logits.size, k, scale, ptr(ids), ptr(w)) == 0
        return ids, w

    def layer_synth(self, policy, seed, layer, ids, w, x, dim, ff, limit=0.0, shared=None):
        ids = np.ascontiguousarray(ids, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        sh = np.ascontiguousarray(shared, np.float32) if shared is not None else None
        y = np.zeros(dim, np.float32)
        rc = self.L.orc_layer_synth(policy, seed, layer, ptr(ids), ptr(w), len(ids), ptr(x),
                                    ptr(sh) if sh is not None else None, dim, ff, limit, ptr(self.scale_table()), 0,
                                    ptr(y))
        assert rc == 0
        return y

    def stack_sensitivity(self, policy, seed, h0, logits, dim, ff, k=6, limit=0.0, first=0):
        """rel_l2 between the stack of h0 and of h0 moved by +-1 ulp (alternating): how far
        any non-bit-exact evaluation order can drift on this input (Q8_K re-quantisation
        between layers turns ulp-level differences into whole quantisation steps)."""
        a = self.stack(policy, seed, h0, logits, dim, ff, k, limit, first)
        h0 = np.ascontiguousarray(h0, np.float32)
        step = np.where(np.arange(h0.size) % 2 == 0, 1, -1).astype(np.int32)
        b = self.stack(policy, seed, (h0.view(np.int32) + step).view(np.float32), logits, dim, ff, k, limit, first)
        return rel_l2(b, a)

    def rmsnorm(self, h):
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros_like(h)
        self.L.orc_rmsnorm(ptr(h), h.size, ptr(out))
        return out

    def stack(self, policy, seed, h0, logits, dim, ff, k=6, limit=0.0, first=0, routes=None):
        """h_{l+1} = h_l + layer_l(RMSNorm(h_l)) with mode-A routing (clb_stack_decode),
        for layers first .. first + len(logits) - 1; routes: optional [(ids, w)] per
        layer used instead of routing the logits."""
        h = np.ascontiguousarray(h0, np.float32).copy()
        for i in range(logits.shape[0]):
            layer = first + i
            ids, w = routes[i] if routes is not None else self.route_sigmoid(logits[i], k)
            y = self.layer_synth(policy, seed, layer, ids, w, self.rmsnorm(h), dim, ff, limit)
            h = (h + y).astype(np.float32)
        return h

    def decode_sub(self, qtype, block, ib):
        q = np.zeros(32, np.int32)
        s = np.zeros(2, np.int32)
        d = C.c_float()
        self.L.orc_decode_sub(qtype, ptr(block), ib, ptr(q), C.byref(d), ptr(s))
        return q, d.value, s

    def integer_lane(self, qtype, block, qblock, lane):
        m, d = C.c_int(), C.c_int()
        self.L.orc_integer_lane(qtype, ptr(block), ptr(qblock), lane, C.byref(m), C.byref(d))
        return m.value, d.value


class Reference:
    """crosslane's own q8k_core.hpp / core.hpp / other_combine.hpp / route.cpp."""

    def __init__(self):
        L = C.CDLL(REF_SO)
        self.L = L
        L.ref_dot.restype = C.c_float
        L.ref_dot.argtypes = [C.c_int, VP, VP, C.c_int]
        L.ref_swiglu.restype = C.c_float
        L.ref_swiglu.argtypes = [C.c_float, C.c_float, C.c_float]
        L.ref_half.restype = C.c_float
        L.ref_half.argtypes = [C.c_uint16]
        L.ref_grid.restype = C.c_uint64
        L.ref_grid.argtypes = [C.c_int, C.c_int]
        L.ref_integer_lane.argtypes = [C.c_int, VP, VP, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.ref_decode_sub.argtypes = [C.c_int, VP, C.c_int, VP, C.POINTER(C.c_float), VP]
        L.ref_combine.argtypes = [VP, VP, C.c_int, VP, VP, C.c_int, VP]
        L.ref_route_cpu.argtypes = [VP, VP, C.c_int, C.c_int, C.c_float, VP, VP]
        L.ref_expert.argtypes = [C.c_int, VP, VP, VP, VP, C.c_int, C.c_int, C.c_float, C.c_int, VP, VP]

    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * Q8K, np.uint8)
        for b in range(x.size // 256):
            self.L.ref_quant_block(ptr(x[256 * b:]), ptr(out[Q8K * b:]))
        return out

    def dot(self, qtype, w_row, q, nb):
        return self.L.ref_dot(qtype, ptr(w_row), ptr(q), nb)

    def integer_lane(self, qtype, block, qblock, lane):
        m, d = C.c_int(), C.c_int()
        self.L.ref_integer_lane(qtype, ptr(block), ptr(qblock), lane, C.byref(m), C.byref(d))
        return m.value, d.value

    def decode_sub(self, qtype, block, ib):
        q = np.zeros(32, np.int32)
        s = np.zeros(2, np.int32)
        d = C.c_float()
        self.L.ref_decode_sub(qtype, ptr(block), ib, ptr(q), C.byref(d), ptr(s))
        return q, d.value, s

    def combine(self, ids, w, rows, shared=None):
        ids = np.ascontiguousarray(ids, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        rows = np.ascontiguousarray(rows, np.float32)
        dim = rows.shape[1]
        out = np.zeros(dim, np.float32)
        sh = np.ascontiguousarray(shared, np.float32) if shared is not None else None
        self.L.ref_combine(ptr(ids), ptr(w), len(ids), ptr(rows), ptr(sh) if sh is not None else None, dim, ptr(out))
        return out

    def route_cpu(self, logits, bias, k, scale):
        logits = np.ascontiguousarray(logits, np.float32)
        bias = np.ascontiguousarray(bias, np.float32)
        ids = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        assert self.L.ref_route_cpu(ptr(logits), ptr(bias), logits.size, k, scale, ptr(ids), ptr(w)) == 0
        return ids, w

    def expert(self, qtype, gate, up, down, x, dim, ff, limit=0.0, threads=0):
        h = np.zeros(ff, np.float32)
        y = np.zeros(dim, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self.L.ref_expert(qtype, ptr(gate), ptr(up), ptr(down), ptr(x), dim, ff, limit, threads, ptr(h), ptr(y))
        return h, y


def reference():
    if not os.path.exists(REF_SO):
        return None
    return Reference()


LANE_SO = os.path.join(os.path.dirname(REF_SO), "..", "liblane.so")


class CpuLane:
    """The timed CPU expert lane (oracle/liblane.so): crosslane's q8k_core.hpp arithmetic
    vectorised with AVX2, layer-batched like the reference lane's Lane::experts."""

    def __init__(self):
        L = C.CDLL(LANE_SO)
        self.L = L
        L.lane_dot.restype = C.c_float
        L.lane_dot.argtypes = [C.c_int, VP, VP, C.c_int]
        L.lane_quantize.argtypes = [VP, C.c_int, VP]
        L.lane_experts.restype = C.c_int
        L.lane_experts.argtypes = [C.c_int, VP, VP, VP, VP, VP, C.c_int, C.c_int, C.c_float, C.c_int, VP]
        L.lane_team_threads.restype = C.c_int
        L.lane_team_threads.argtypes = [C.c_int]

    def dot(self, qtype, w_row, q, nb):
        return self.L.lane_dot(qtype, ptr(w_row), ptr(q), nb)

    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * Q8K, np.uint8)
        self.L.lane_quantize(ptr(x), x.size, ptr(out))
        return out

    def experts(self, types, gates, ups, downs, x, dim, ff, limit=0.0, threads=0):
        """y [n][dim] of n experts (ggml AoS matrices) on one x; returns (y, team size)."""
        n = len(types)
        t = np.ascontiguousarray(types, np.int32)
        arr = lambda ms: (C.c_void_p * n)(*[m.ctypes.data for m in ms])
        g, u, d = arr(gates), arr(ups), arr(downs)
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros((n, dim), np.float32)
        used = self.L.lane_experts(n, ptr(t), C.cast(g, VP), C.cast(u, VP), C.cast(d, VP), ptr(x), dim, ff, limit,
                                   threads, ptr(y))
        return y, used


def cpu_lane():
    return CpuLane() if os.path.exists(LANE_SO) else None


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs_rel(a, b):
    """max |a - b| / max |b| (the max-abs-relative metric of the parity contract)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def tie_probe(n):
    """Every 256-block: element 0 = 127, others half-integers: Q8_K scale exactly 1 and
    exact .5 rounding ties (crosslane engine/tools/strata-p1k/iq_probe.hpp:6-13, on 256 blocks)."""
    x = np.zeros(n, np.float32)
    for i in range(n):
        x[i] = 127.0 if i % 256 == 0 else float((i % 31) - 15) + 0.5
    return x
