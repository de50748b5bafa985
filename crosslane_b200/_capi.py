"""ctypes binding of include/crosslane_b200.h (libcrosslane_b200.so).

There is no fallback: if the shared library is missing or fails to load, importing
this module raises, so nothing can silently run a non-CUDA path.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# CROSSLANE_B200_LIB selects another build of the library (e.g. the phase-trace build);
# the default is the in-tree libcrosslane_b200.so.
LIB_PATH = os.environ.get("CROSSLANE_B200_LIB") or os.path.join(_HERE, "libcrosslane_b200.so")

CLB_OK = 0
CLB_E_INVALID = 1
CLB_E_CUDA = 2
CLB_E_NOMEM = 3
CLB_E_STATE = 4
CLB_E_NONFINITE = 5
CLB_E_UNSUPPORTED = 6
CLB_E_LANE = 7
CLB_E_NCCL = 8

ERROR_NAMES = {0: "CLB_OK", 1: "CLB_E_INVALID", 2: "CLB_E_CUDA", 3: "CLB_E_NOMEM", 4: "CLB_E_STATE",
               5: "CLB_E_NONFINITE", 6: "CLB_E_UNSUPPORTED", 7: "CLB_E_LANE", 8: "CLB_E_NCCL"}


class ClbError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


class TimingV1(C.Structure):
    _fields_ = [("ns", C.c_uint64), ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64), ("layer", C.c_int32),
                ("layers", C.c_int32), ("picks", C.c_int32), ("reserved", C.c_int32)]


class LaneConfigV1(C.Structure):
    _fields_ = [("experts", C.c_int32), ("exact_math", C.c_int32), ("bytes", C.c_uint64), ("device_first", C.c_int32),
                ("device_last", C.c_int32), ("timing", C.c_int32), ("bank_flags", C.c_int32),
                ("reserved", C.c_int32 * 6)]


class ErrorV1(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char * 512)]


class BankConfigV1(C.Structure):
    _fields_ = [("device", C.c_int32), ("n_layers", C.c_int32), ("n_experts", C.c_int32), ("dim", C.c_int32),
                ("ff", C.c_int32), ("max_picks", C.c_int32), ("limit", C.c_float), ("expert_begin", C.c_int32),
                ("expert_end", C.c_int32), ("flags", C.c_int32),
                ("reserved", C.c_int32 * 6)]


HOST_EXPERT_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_uint32, C.c_int32, C.POINTER(C.c_float), C.c_int32,
                             C.POINTER(C.c_float))

_P = C.c_void_p
_I = C.c_int32
_U32 = C.c_uint32
_F = C.c_float
_SZ = C.c_size_t
_PE = C.POINTER(ErrorV1)

# name: (restype, argtypes)
SIGNATURES = {
    "clb_abi_version": (_I, []),
    "clb_q8k_activation_bytes": (_SZ, [_I]),
    "clb_q8k_quantize": (_I, [_P, _P, _I, _P]),
    "clb_q8k_mv": (_I, [_I, _P, _P, _P, _I, _I, _P]),
    "clb_q8k_activate": (_I, [_P, _P, _P, _I, _F, _P]),
    "clb_decode_tables": (_SZ, [_P, _SZ]),
    "clb_packed_bytes": (_SZ, [_I, _I, _I]),
    "clb_pack": (_I, [_I, _I, _I, _P, _SZ, _P, _SZ]),
    "clb_unpack": (_I, [_I, _I, _I, _P, _SZ, _P, _SZ]),
    "clb_bank_create": (_I, [C.POINTER(BankConfigV1), C.POINTER(_P), _PE]),
    "clb_bank_destroy": (None, [_P]),
    "clb_bank_fill_synthetic": (_I, [_P, C.c_uint64, _I, _PE]),
    "clb_bank_load_matrix": (_I, [_P, _U32, _I, _I, _I, _P, _SZ, _PE]),
    "clb_bank_weight_bytes": (C.c_uint64, [_P]),
    "clb_bank_stack_persistent": (_I, [_P]),
    "clb_bank_set_wait_limit": (_I, [_P, C.c_uint32, _PE]),
    "clb_bank_exchange_handle": (_I, [_P, _P, _PE]),
    "clb_bank_connect": (_I, [_P, _I, _I, _P, _PE]),
    "clb_placement_parse": (_I, [C.c_char_p, _SZ, _I, _I, _P, C.POINTER(C.c_uint64), _PE]),
    "clb_bank_apply_placement": (_I, [_P, _P, _I, _PE]),
    "clb_bank_placed": (_I, [_P, _U32, _I]),
    "clb_strata_pack_open": (_I, [C.c_char_p, C.POINTER(_P), _PE]),
    "clb_strata_pack_close": (None, [_P]),
    "clb_strata_pack_meta": (_I, [_P, C.c_char_p, C.c_char_p, _SZ]),
    "clb_strata_pack_tensor": (_I, [_P, C.c_char_p, C.c_char_p, _SZ, C.POINTER(C.c_uint64), C.POINTER(C.c_int64), _I,
                                    C.POINTER(_I)]),
    "clb_strata_pack_read": (_I, [_P, C.c_char_p, C.c_uint64, _P, C.c_uint64, _PE]),
    "clb_bank_load_strata_pack": (_I, [_P, _P, _U32, _PE]),
    "clb_bank_geometry": (_I, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_I), C.POINTER(_I)]),
    "clb_bank_contains": (_I, [_P, _U32, _I]),
    "clb_bank_compute": (_I, [_P, _U32, _I, _P, _P, _PE]),
    "clb_bank_compute_many": (_I, [_P, _U32, _P, _I, _P, _P, _PE]),
    "clb_layer_execute": (_I, [_P, _U32, _P, _P, _I, _P, _P, _P, _PE]),
    "clb_layer_forward_device": (_I, [_P, _U32, _P, _P, _I, _P, _P, _P, _P, _P, _PE]),
    "clb_layer_phases_device": (_I, [_P, _U32, _P, _P, _I, _P, _P, _I, _P, _PE]),
    "clb_bank_expert_info": (_I, [_P, _U32, _I, C.POINTER(_I), C.POINTER(C.c_uint64)]),
    "clb_route_device": (_I, [_I, _P, _I, _I, _I, _P, _P, _P]),
    "clb_route_host": (_I, [_I, _P, _P, _I, _I, _F, _P, _P]),
    "clb_router_device": (_I, [_P, _I, _I, _P, _I, _P, _P]),
    "clb_route_b_device": (_I, [_P, _P, _I, _I, _I, _F, _P, _P, _P, _P]),
    "clb_moe_block_device": (_I, [_P, _U32, _P, _P, _P, _F, _P, _P, _P, _P, _P, _P, _P, _PE]),
    "clb_stack_decode": (_I, [_P, _U32, _I, _P, _P, _P, _PE]),
    "clb_stack_decode_device": (_I, [_P, _U32, _I, _P, _P, _PE]),
    "clb_prefill_workspace_bytes": (C.c_uint64, [_P, _I, _I]),
    "clb_prefill_layer_device": (_I, [_P, _U32, _I, _I, _P, _P, _P, _P, _P, _P, C.c_uint64, _P, _PE]),
    "clb_prefill_phases_device": (_I, [_P, _U32, _I, _I, _P, _P, _P, _P, _P, C.c_uint64, _I, _P, _PE]),
    "clb_prefill_reserve": (_I, [_P, _I, _I, _PE]),
    "clb_prefill_layer": (_I, [_P, _U32, _I, _I, _P, _P, _P, _P, _PE]),
    "clb_stack_batch_workspace_bytes": (C.c_uint64, [_P, _I]),
    "clb_stack_batch_device": (_I, [_P, _U32, _I, _I, _P, _P, _P, C.c_uint64, _P, _PE]),
    "clb_stack_batch": (_I, [_P, _U32, _I, _I, _P, _P, _PE]),
    "clb_stack_batch_layer_device": (_I, [_P, _U32, _I, _P, _P, _P, _P, C.c_uint64, _I, _P, _PE]),
    "clb_bank_stream": (_P, [_P]),
    "clb_bank_last_timing": (_I, [_P, _P]),
    "clb_lane_config_parse": (_I, [C.c_char_p, _P, _PE]),
    "clb_bank_synchronize": (_I, [_P, _PE]),
    "clb_warm_execute": (_I, [_P, _U32, _P, _P, _I, _P, _P, HOST_EXPERT_FN, _P, _P, _PE]),
    "clb_expert_forward_noalloc": (_I, [_I, _P, _P, _P, _P, _P, _I, _I, _F, _P, _PE]),
}


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise ImportError(f"crosslane_b200: CUDA library {path} is not built "
                          "(run `python crosslane_b200/build.py`); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load()


def check(rc: int, err: ErrorV1 = None, what: str = ""):
    if rc != CLB_OK:
        msg = err.message.decode(errors="replace") if err is not None else what
        raise ClbError(rc, msg or what)
