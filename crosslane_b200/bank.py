"""Python face of the CUDA expert lane.

`ExpertBank` mirrors crosslane's expert-lane interface `WarmRedirect`
(engine/strata/warm/runtime.hpp:10-16): warm_contains / warm_grouped / warm_compute /
warm_compute_many, plus `warm_execute` (engine/strata/warm/runtime.cpp:121-189) with a
host lane for non-resident experts. Every call goes through the C ABI in
include/crosslane_b200.h; host arrays are numpy float32, device arrays torch tensors.
"""
import ctypes as C

import numpy as np

from . import _capi
from ._capi import BankConfigV1, ErrorV1, HOST_EXPERT_FN, LaneConfigV1, TimingV1, check, lib

IQ2_XXS, IQ2_XS, IQ1_M = 16, 17, 29
BLOCK_BYTES = {IQ2_XXS: 66, IQ2_XS: 74, IQ1_M: 56}
EXACT_ORDER = 1  # CLB_BANK_EXACT_ORDER
PER_LAYER_KERNELS = 2  # CLB_BANK_PER_LAYER_KERNELS
TIMING = 4  # CLB_BANK_TIMING
EXCHANGE_HANDLE_BYTES = 64  # CLB_EXCHANGE_HANDLE_BYTES
ROLE_GATE, ROLE_UP, ROLE_DOWN = 0, 1, 2
Q8K_BLOCK_BYTES = 292


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _stream(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(stream)


class ExpertBank:
    """A resident bank of routed experts on one GPU (the CUDA lane)."""

    def __init__(self, *, n_layers: int, n_experts: int, dim: int, ff: int, max_picks: int = 6,
                 limit: float = 0.0, device: int = 0, expert_begin: int = 0, expert_end: int = 0,
                 exact_order: bool = False, per_layer_kernels: bool = False, timing: bool = False):
        flags = ((EXACT_ORDER if exact_order else 0) | (PER_LAYER_KERNELS if per_layer_kernels else 0) |
                 (TIMING if timing else 0))
        cfg = BankConfigV1(device=device, n_layers=n_layers, n_experts=n_experts, dim=dim, ff=ff,
                           max_picks=max_picks, limit=limit, expert_begin=expert_begin, expert_end=expert_end,
                           flags=flags)
        err = ErrorV1()
        h = C.c_void_p()
        check(lib.clb_bank_create(C.byref(cfg), C.byref(h), C.byref(err)), err)
        self._h = h
        self.n_layers, self.n_experts, self.dim, self.ff = n_layers, n_experts, dim, ff
        self.max_picks, self.limit, self.device = max_picks, limit, device
        self.expert_begin = expert_begin
        self.expert_end = expert_end or n_experts

    # -- lifetime --
    def close(self):
        if getattr(self, "_h", None):
            lib.clb_bank_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- loading --
    def fill_synthetic(self, seed: int, type_policy: int) -> None:
        err = ErrorV1()
        check(lib.clb_bank_fill_synthetic(self._h, C.c_uint64(seed), type_policy, C.byref(err)), err)

    def load_matrix(self, layer: int, expert: int, role: int, qtype: int, ggml: np.ndarray) -> None:
        buf = np.ascontiguousarray(ggml, dtype=np.uint8)
        err = ErrorV1()
        check(lib.clb_bank_load_matrix(self._h, layer, expert, role, qtype, _ptr(buf), buf.nbytes, C.byref(err)), err)

    def set_wait_limit(self, polls: int) -> None:
        """Polls before a stack kernel's bounded device wait gives up (CLB_E_CUDA, bank poisoned)."""
        err = ErrorV1()
        check(lib.clb_bank_set_wait_limit(self._h, polls, C.byref(err)), err)

    @property
    def persistent(self) -> bool:
        """Stack decode runs as the persistent kernel (else the per-layer kernels)."""
        return bool(lib.clb_bank_stack_persistent(self._h))

    @property
    def weight_bytes(self) -> int:
        return int(lib.clb_bank_weight_bytes(self._h))

    @property
    def stream(self) -> int:
        return int(lib.clb_bank_stream(self._h) or 0)

    def synchronize(self) -> None:
        err = ErrorV1()
        check(lib.clb_bank_synchronize(self._h, C.byref(err)), err)

    # -- WarmRedirect --
    def warm_grouped(self) -> bool:
        return True

    def warm_contains(self, layer: int, expert: int) -> bool:
        return bool(lib.clb_bank_contains(self._h, layer, expert))

    def warm_compute(self, layer: int, expert: int, x) -> np.ndarray:
        x = _f32(x)
        y = np.empty(self.dim, np.float32)
        err = ErrorV1()
        check(lib.clb_bank_compute(self._h, layer, expert, _ptr(x), _ptr(y), C.byref(err)), err)
        return y

    def warm_compute_many(self, layer: int, ids, x) -> np.ndarray:
        ids = _i32(ids)
        x = _f32(x)
        y = np.empty((len(ids), self.dim), np.float32)
        err = ErrorV1()
        check(lib.clb_bank_compute_many(self._h, layer, _ptr(ids), len(ids), _ptr(x), _ptr(y), C.byref(err)), err)
        return y

    # -- frozen warm placement (crosslane_b200.placement) --
    def apply_placement(self, lanes, lane_id: int = 3) -> None:
        """Hold exactly the experts `lanes` [layers][experts] assigns to `lane_id` (3 = CUDA,
        or 1 = the GPU-lane slot); before any weights are loaded."""
        lanes = np.ascontiguousarray(lanes, dtype=np.int32)
        assert lanes.shape == (self.n_layers, self.n_experts)
        err = ErrorV1()
        check(lib.clb_bank_apply_placement(self._h, _ptr(lanes), lane_id, C.byref(err)), err)

    def load_strata_pack(self, pack, first_layer: int = 0) -> None:
        """Repack every matrix placed on this bank from a crosslane_b200.strata_pack.StrataPack
        (bank layer l <- pack layer first_layer + l)."""
        err = ErrorV1()
        check(lib.clb_bank_load_strata_pack(self._h, pack.handle, first_layer, C.byref(err)), err)

    def placed(self, layer: int, expert: int) -> bool:
        return bool(lib.clb_bank_placed(self._h, layer, expert))

    # -- layer / stack --
    def layer_execute(self, layer: int, ids, w, x, shared=None) -> np.ndarray:
        ids, w, x = _i32(ids), _f32(w), _f32(x)
        sh = _f32(shared) if shared is not None else None
        out = np.empty(self.dim, np.float32)
        err = ErrorV1()
        check(lib.clb_layer_execute(self._h, layer, _ptr(ids), _ptr(w), len(ids), _ptr(x),
                                    _ptr(sh) if sh is not None else None, _ptr(out), C.byref(err)), err)
        return out

    def warm_execute(self, layer: int, ids, w, x, shared=None, host_lane=None) -> np.ndarray:
        """host_lane(layer, expert, x: np.ndarray) -> np.ndarray[dim] for non-resident picks."""
        ids, w, x = _i32(ids), _f32(w), _f32(x)
        sh = _f32(shared) if shared is not None else None
        out = np.empty(self.dim, np.float32)
        dim = self.dim

        def trampoline(_ctx, layer_, expert, xp, n, yp):
            try:
                xv = np.ctypeslib.as_array(xp, shape=(n,)).copy()
                y = np.asarray(host_lane(layer_, expert, xv), dtype=np.float32)
                if y.shape != (dim,):
                    return 1
                C.memmove(yp, y.ctypes.data, 4 * dim)
                return 0
            except Exception:
                return 1

        cb = HOST_EXPERT_FN(trampoline) if host_lane is not None else HOST_EXPERT_FN()
        err = ErrorV1()
        check(lib.clb_warm_execute(self._h, layer, _ptr(ids), _ptr(w), len(ids), _ptr(x),
                                   _ptr(sh) if sh is not None else None, cb, None, _ptr(out), C.byref(err)), err)
        return out

    def stack_decode(self, first_layer: int, n_layers: int, x, logits) -> np.ndarray:
        x = _f32(x)
        logits = _f32(logits)
        assert logits.shape == (n_layers, self.n_experts)
        out = np.empty(self.dim, np.float32)
        err = ErrorV1()
        check(lib.clb_stack_decode(self._h, first_layer, n_layers, _ptr(x), _ptr(logits), _ptr(out), C.byref(err)),
              err)
        return out

    # -- expert-ID sharding over GPUs (clb_bank_exchange_handle / clb_bank_connect) --
    def exchange_handle(self) -> bytes:
        """CUDA IPC handle (64 bytes) of this bank's exchange region, for the peer processes."""
        buf = (C.c_ubyte * EXCHANGE_HANDLE_BYTES)()
        err = ErrorV1()
        check(lib.clb_bank_exchange_handle(self._h, buf, C.byref(err)), err)
        return bytes(buf)

    def connect(self, rank: int, world: int, handles) -> None:
        """Open the peers' exchange regions; handles[r] is rank r's exchange_handle()."""
        blob = b"".join(bytes(h) for h in handles)
        assert len(blob) == world * EXCHANGE_HANDLE_BYTES
        buf = (C.c_ubyte * len(blob)).from_buffer_copy(blob)
        err = ErrorV1()
        check(lib.clb_bank_connect(self._h, rank, world, buf, C.byref(err)), err)

    def stack_decode_device(self, first_layer: int, n_layers: int, d_x, d_logits) -> None:
        """d_x: torch float32 [dim] on this device, updated in place on the bank stream."""
        err = ErrorV1()
        check(lib.clb_stack_decode_device(self._h, first_layer, n_layers, C.c_void_p(d_x.data_ptr()),
                                          C.c_void_p(d_logits.data_ptr()), C.byref(err)), err)

    def layer_phases_device(self, layer: int, d_ids, d_w, d_x, d_out, phase_mask: int, stream=None) -> None:
        err = ErrorV1()
        check(lib.clb_layer_phases_device(
            self._h, layer, C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_w.data_ptr()), d_ids.numel(),
            C.c_void_p(d_x.data_ptr()), C.c_void_p(d_out.data_ptr()), phase_mask,
            C.c_void_p(stream) if stream else None, C.byref(err)), err)

    # -- batched prefill (clb_prefill_*) --
    def prefill_workspace_bytes(self, tokens: int, k: int) -> int:
        return int(lib.clb_prefill_workspace_bytes(self._h, tokens, k))

    def prefill_reserve(self, tokens: int, k: int) -> None:
        err = ErrorV1()
        check(lib.clb_prefill_reserve(self._h, tokens, k, C.byref(err)), err)

    def prefill_layer(self, layer: int, ids, w, x) -> np.ndarray:
        """ids/w [T][k], x [T][dim] host arrays -> out [T][dim] (synchronous)."""
        ids, w, x = _i32(ids), _f32(w), _f32(x)
        T, k = ids.shape
        assert w.shape == (T, k) and x.shape == (T, self.dim)
        out = np.empty((T, self.dim), np.float32)
        err = ErrorV1()
        check(lib.clb_prefill_layer(self._h, layer, T, k, _ptr(ids), _ptr(w), _ptr(x), _ptr(out), C.byref(err)), err)
        return out

    def prefill_layer_device(self, layer: int, d_ids, d_w, d_x, d_out, d_ws, d_resid=None, stream=None) -> None:
        """torch tensors on this device: d_ids int32 [T][k], d_w [T][k], d_x/d_out [T][dim],
        d_ws uint8 workspace (prefill_workspace_bytes); runs on the bank stream."""
        T, k = d_ids.shape
        err = ErrorV1()
        check(lib.clb_prefill_layer_device(
            self._h, layer, T, k, C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_w.data_ptr()),
            C.c_void_p(d_x.data_ptr()), C.c_void_p(d_resid.data_ptr()) if d_resid is not None else None,
            C.c_void_p(d_out.data_ptr()), C.c_void_p(d_ws.data_ptr()), d_ws.numel(),
            C.c_void_p(stream) if stream else None, C.byref(err)), err)

    def prefill_phases_device(self, layer: int, d_ids, d_w, d_x, d_out, d_ws, phase_mask: int, stream=None) -> None:
        T, k = d_ids.shape
        err = ErrorV1()
        check(lib.clb_prefill_phases_device(
            self._h, layer, T, k, C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_w.data_ptr()),
            C.c_void_p(d_x.data_ptr()), C.c_void_p(d_out.data_ptr()), C.c_void_p(d_ws.data_ptr()), d_ws.numel(),
            phase_mask, C.c_void_p(stream) if stream else None, C.byref(err)), err)

    # -- batched stack decode (clb_stack_batch*) --
    def stack_batch_workspace_bytes(self, tokens: int) -> int:
        return int(lib.clb_stack_batch_workspace_bytes(self._h, tokens))

    def stack_batch(self, first_layer: int, n_layers: int, h, logits) -> np.ndarray:
        """h [T][dim], logits [n_layers][T][n_experts] host arrays -> h after the layers
        (synchronous; routing on the host)."""
        h, logits = _f32(h).copy(), _f32(logits)
        T = h.shape[0]
        assert h.shape == (T, self.dim) and logits.shape == (n_layers, T, self.n_experts)
        err = ErrorV1()
        check(lib.clb_stack_batch(self._h, first_layer, n_layers, T, _ptr(logits), _ptr(h), C.byref(err)), err)
        return h

    def stack_batch_device(self, first_layer: int, n_layers: int, d_h, d_logits, d_ws, stream=None) -> None:
        """torch tensors on this device: d_h [T][dim] (updated in place), d_logits
        [n_layers][T][n_experts], d_ws uint8 (stack_batch_workspace_bytes); routing on the device."""
        err = ErrorV1()
        check(lib.clb_stack_batch_device(
            self._h, first_layer, n_layers, d_h.shape[0], C.c_void_p(d_logits.data_ptr()), C.c_void_p(d_h.data_ptr()),
            C.c_void_p(d_ws.data_ptr()), d_ws.numel(), C.c_void_p(stream) if stream else None, C.byref(err)), err)

    def stack_batch_layer_device(self, layer: int, d_h, d_logits, d_rows, d_ws, phase_mask: int, stream=None) -> None:
        """One layer of the batched stack (clb_stack_batch_layer_device): phase bit 1 computes
        this bank's expert rows into d_rows [T*k][dim], bit 2 adds the combine of d_rows to d_h."""
        err = ErrorV1()
        check(lib.clb_stack_batch_layer_device(
            self._h, layer, d_h.shape[0], C.c_void_p(d_logits.data_ptr()), C.c_void_p(d_h.data_ptr()),
            C.c_void_p(d_rows.data_ptr()), C.c_void_p(d_ws.data_ptr()), d_ws.numel(), phase_mask,
            C.c_void_p(stream) if stream else None, C.byref(err)), err)

    def moe_block_device(self, layer: int, d_x, d_gate_w, d_bias, scale: float, d_out, d_logits, d_ids, d_w,
                         d_shared=None, d_resid=None, stream=None) -> None:
        """Router + route_cpu + experts + combine of one token on the device (clb_moe_block_device)."""
        err = ErrorV1()
        vp = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
        check(lib.clb_moe_block_device(self._h, layer, vp(d_x), vp(d_gate_w), vp(d_bias), scale, vp(d_shared),
                                       vp(d_resid), vp(d_out), vp(d_logits), vp(d_ids), vp(d_w),
                                       C.c_void_p(stream) if stream else None, C.byref(err)), err)

    def last_timing(self) -> dict:
        """The last CLB_BANK_TIMING span (clb_bank_last_timing) as a dict."""
        t = TimingV1()
        check(lib.clb_bank_last_timing(self._h, C.byref(t)), what="clb_bank_last_timing")
        return {f: getattr(t, f) for f, _ in TimingV1._fields_ if f != "reserved"}

    def expert_info(self, layer: int, expert: int):
        """(ggml type id, payload bytes of gate+up+down) of a resident expert."""
        t = C.c_int32()
        b = C.c_uint64()
        check(lib.clb_bank_expert_info(self._h, layer, expert, C.byref(t), C.byref(b)), what="not resident")
        return int(t.value), int(b.value)

    def layer_forward_device(self, layer: int, d_ids, d_w, d_x, d_out, d_shared=None, d_resid=None,
                             stream=None) -> None:
        err = ErrorV1()
        check(lib.clb_layer_forward_device(
            self._h, layer, C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_w.data_ptr()), d_ids.numel(),
            C.c_void_p(d_x.data_ptr()), C.c_void_p(d_shared.data_ptr()) if d_shared is not None else None,
            C.c_void_p(d_resid.data_ptr()) if d_resid is not None else None, C.c_void_p(d_out.data_ptr()),
            C.c_void_p(stream) if stream else None, C.byref(err)), err)


# -- stateless primitives ------------------------------------------------------------

def packed_bytes(qtype: int, n: int, k: int) -> int:
    return int(lib.clb_packed_bytes(qtype, n, k))


def pack(qtype: int, n: int, k: int, ggml: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(ggml, dtype=np.uint8)
    out = np.zeros(packed_bytes(qtype, n, k), np.uint8)
    check(lib.clb_pack(qtype, n, k, _ptr(src), src.nbytes, _ptr(out), out.nbytes), what="clb_pack")
    return out


def unpack(qtype: int, n: int, k: int, packed: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros(n * (k // 256) * BLOCK_BYTES[qtype], np.uint8)
    check(lib.clb_unpack(qtype, n, k, _ptr(src), src.nbytes, _ptr(out), out.nbytes), what="clb_unpack")
    return out


def route_host(mode: int, logits, k: int, bias=None, scale: float = 1.0):
    logits = _f32(logits)
    b = _f32(bias) if bias is not None else None
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    check(lib.clb_route_host(mode, _ptr(logits), _ptr(b) if b is not None else None, logits.size, k, scale,
                             _ptr(ids), _ptr(w)), what="clb_route_host")
    return ids, w


def q8k_quantize(d_x, d_q, stream=None) -> None:
    check(lib.clb_q8k_quantize(C.c_void_p(d_x.data_ptr()), C.c_void_p(d_q.data_ptr()), d_x.numel(),
                               _stream(stream)), what="clb_q8k_quantize")


def q8k_mv(qtype: int, d_w, d_q, d_y, n: int, k: int, stream=None) -> None:
    check(lib.clb_q8k_mv(qtype, C.c_void_p(d_w.data_ptr()), C.c_void_p(d_q.data_ptr()), C.c_void_p(d_y.data_ptr()),
                         n, k, _stream(stream)), what="clb_q8k_mv")


def q8k_activate(d_g, d_u, d_h, limit: float = 0.0, stream=None) -> None:
    check(lib.clb_q8k_activate(C.c_void_p(d_g.data_ptr()), C.c_void_p(d_u.data_ptr()), C.c_void_p(d_h.data_ptr()),
                               d_g.numel(), limit, _stream(stream)), what="clb_q8k_activate")


def route_device(d_logits, n_experts: int, k: int, tokens: int, d_ids, d_w, stream=None) -> None:
    check(lib.clb_route_device(0, C.c_void_p(d_logits.data_ptr()), n_experts, k, tokens, C.c_void_p(d_ids.data_ptr()),
                               C.c_void_p(d_w.data_ptr()), _stream(stream)), what="clb_route_device")


def router_device(d_x, d_gate_w, d_logits, stream=None) -> None:
    """d_logits [T][E] = d_gate_w [E][dim] . d_x [T][dim] (fp32, torch tensors on the device)."""
    T, dim = d_x.shape
    check(lib.clb_router_device(C.c_void_p(d_x.data_ptr()), T, dim, C.c_void_p(d_gate_w.data_ptr()),
                                d_gate_w.shape[0], C.c_void_p(d_logits.data_ptr()), _stream(stream)),
          what="clb_router_device")


def route_b_device(d_logits, d_bias, k: int, scale: float, d_ids, d_w, d_status, stream=None) -> None:
    """route_cpu on the device: d_logits [T][E], d_bias [E] -> d_ids/d_w [T][k]; d_status int32 [1]."""
    T, E = d_logits.shape
    check(lib.clb_route_b_device(C.c_void_p(d_logits.data_ptr()), C.c_void_p(d_bias.data_ptr()), E, k, T, scale,
                                 C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_w.data_ptr()),
                                 C.c_void_p(d_status.data_ptr()), _stream(stream)), what="clb_route_b_device")


def lane_config_parse(text: str) -> dict:
    """The CUDA lane's keys of a stage config (clb_lane_config_parse) as a dict; raises
    ClbError on a malformed, duplicate or unknown key."""
    c = LaneConfigV1()
    err = ErrorV1()
    check(lib.clb_lane_config_parse(text.encode(), C.byref(c), C.byref(err)), err)
    return {f: getattr(c, f) for f, _ in LaneConfigV1._fields_ if f != "reserved"}
