"""crosslane_b200: B200-native (sm_100a) routed-expert decode lane for crosslane.

The product is the C ABI in include/crosslane_b200.h, implemented by
libcrosslane_b200.so (CUDA kernels + C++ host runtime). This package binds it for
Python callers; importing it fails if the library is not built.
"""
from ._capi import ClbError, lib  # noqa: F401  (raises ImportError if the .so is missing)
from .bank import (BLOCK_BYTES, IQ1_M, IQ2_XS, IQ2_XXS, Q8K_BLOCK_BYTES, ROLE_DOWN, ROLE_GATE,  # noqa: F401
                   ROLE_UP, ExpertBank, lane_config_parse, pack, packed_bytes, q8k_activate, q8k_mv, q8k_quantize,
                   route_b_device, route_device, route_host, router_device, unpack)

__all__ = ["ExpertBank", "ClbError", "pack", "unpack", "packed_bytes", "route_host", "route_device",
           "router_device", "route_b_device", "lane_config_parse",
           "q8k_quantize", "q8k_mv", "q8k_activate", "IQ2_XXS", "IQ2_XS", "IQ1_M", "BLOCK_BYTES",
           "ROLE_GATE", "ROLE_UP", "ROLE_DOWN", "Q8K_BLOCK_BYTES"]
