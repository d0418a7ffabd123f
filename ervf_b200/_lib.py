"""ctypes binding of libervf_b200.so (the C ABI in include/ervf_b200.h).

The library is the only compute path of this package: if it is missing or
fails to load, every entry point raises -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libervf_b200.so"

OK = 0
ERR_NULL = -1
ERR_SHAPE = -2
ERR_ALIGN = -3
ERR_LAUNCH = -4
ERR_TIMEOUT = -5
ERR_ARG = -6
ERR_DEVICE = -7
ERR_SCRATCH_LIMIT = -8

LAUNCH_PDL = 1
LAUNCH_IDS_READY = 2
UP_SWIGLU = 4

_NAMES = {
    ERR_NULL: "null pointer",
    ERR_SHAPE: "unsupported shape",
    ERR_ALIGN: "misaligned pointer or stride",
    ERR_LAUNCH: "CUDA launch failed",
    ERR_TIMEOUT: "device wait timed out",
    ERR_ARG: "invalid argument",
    ERR_DEVICE: "CUDA set-up call failed",
    ERR_SCRATCH_LIMIT: "larger than the fixed scratch array (hidden <= 8192, top_k <= 8)",
}

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> argtypes (all return int)
SIGNATURES: dict[str, list] = {
    "ervf_version": [],
    "ervf_device_status": [],
    "ervf_nvfp4_gemv": [_vp, _vp, _vp, _vp, _f, _i, _i, _i, _f, _i, _i, _vp],
    "ervf_nvfp4_gemv_ind": [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _f, _sz, _sz, _i, _vp],
    "ervf_nvfp4_gemv_grouped": [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _vp],
    "ervf_weighted_accumulate": [_vp, _vp, _f, _i, _vp],
    "ervf_weighted_accumulate_ind": [_vp, _vp, _vp, _i, _vp],
    "ervf_moe_up_grouped": [_vp, _vp, _sz, _sz, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _vp],
    "ervf_moe_down_routesum": [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i,
                               _vp, _sz, _i, _i, _vp],
    "ervf_routesum_scratch_bytes": [_i, _i],
    "ervf_moe_layer": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i,
                       _i, _i, _vp, _sz, _vp, _vp, _vp, _i, _vp],
    "ervf_moe_token": [_vp, _i, _sz, _sz, _sz, _sz, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _vp, _sz, _i,
                       _vp],
    "ervf_moe_token_scratch_bytes": [_i, _i, _i, _i],
    "ervf_moe_token_ep": [_vp, _i, _sz, _sz, _sz, _sz, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _vp, _i,
                          _i, _sz, _i, _i, _vp],
    "ervf_moe_token_ep_scratch_bytes": [_i, _i, _i, _i],
    "ervf_moe_token_ep_prepare": [_vp, _sz, _i, _i, _i, _i, _vp],
    "ervf_moe_token_router": [_vp, _i, _sz, _sz, _sz, _sz, _vp, _vp, _i, _i, _f, _i, _vp, _vp, _i, _i,
                              _vp, _sz, _i, _vp],
    "ervf_moe_down_routesum_static": [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp,
                                      _i, _i, _i, _i, _vp],
    "ervf_moe_batched": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _vp, _i, _i, _i, _vp, _vp,
                         _i, _i, _vp, _sz, _vp],
    "ervf_moe_batched_scratch_bytes": [_i, _i, _i, _i],
    "ervf_moe_batched_ex": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _vp, _i, _i, _i, _vp,
                            _vp, _i, _i, _i, _i, _vp, _sz, _vp],
    "ervf_moe_batched_ep_slots_ex": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _i, _i, _i,
                                     _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp],
    "ervf_moe_batched_ep_slots": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _i, _i, _i,
                                  _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp],
    "ervf_ep_batch_exchange_route_sum": [_vp, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _i, _i, _vp,
                                         _sz, _i, _vp],
    "ervf_bf16_gemm_tc": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ervf_nvfp4_gemm_tc": [_vp, _vp, _f, _vp, _vp, _i, _i, _i, _vp, _sz, _vp],
    "ervf_nvfp4_gemm_tc_scratch_bytes": [_i, _i, _i],
    "ervf_route_topk_softmax": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ervf_route_topk_batched": [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp],
    "ervf_ep_expert_slots": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _i, _vp, _vp, _vp,
                             _i, _i, _i, _i, _i, _vp],
    "ervf_ep_route_sum": [_vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp],
    "ervf_ep_expert_slots_ex": [_vp, _vp, _sz, _sz, _vp, _vp, _sz, _sz, _vp, _vp, _i, _vp, _vp,
                                _vp, _i, _i, _i, _i, _i, _i, _vp],
    "ervf_ep_region_bytes": [_i, _i],
    "ervf_ep_region_alloc": [_sz, _vp, _vp],
    "ervf_ep_region_open": [_vp, _vp],
    "ervf_ep_region_close": [_vp],
    "ervf_ep_region_free": [_vp],
    "ervf_ep_exchange_route_sum": [_vp, _i, _i, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _vp],
    "ervf_down_masked": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp],
    "ervf_down_masked_ind": [_vp, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp],
    "ervf_panel_major": [_vp, _vp, _vp, _i, _i, _vp],
    "ervf_bf16_gemv": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ervf_nvfp4_gemm_rows_b": [_vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp, _vp],
    "ervf_down_union": [_vp, _vp, _i, _vp, _vp, _f, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                        _vp],
    "ervf_reduce_slots": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ervf_route_topk": [_vp, _vp, _vp, _vp, _i, _i, _f, _i, _vp],
    "ervf_f32_gemv": [_vp, _vp, _vp, _i, _i, _vp],
    "ervf_route_gemv_topk": [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _vp, _i, _vp],
    "ervf_cache_assign": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp],
    "ervf_cache_fetch": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _i, _vp],
}

SIZE_RESULT = {"ervf_routesum_scratch_bytes", "ervf_nvfp4_gemm_tc_scratch_bytes",
               "ervf_moe_token_scratch_bytes", "ervf_moe_token_ep_scratch_bytes",
               "ervf_moe_batched_scratch_bytes", "ervf_ep_region_bytes"}

_lib = None


class ErvfError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {_NAMES.get(status, 'status')} ({status})")
        self.status = status


def load():
    """Load (once) and return the ctypes library; raise if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m ervf_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL | getattr(os, "RTLD_NOW", 2))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_size_t if name in SIZE_RESULT else ctypes.c_int
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Call one C entry point and raise ErvfError on a non-zero status."""
    status = getattr(load(), name)(*args)
    if status != OK:
        if status in (ERR_SHAPE, ERR_ALIGN, ERR_ARG, ERR_NULL, ERR_SCRATCH_LIMIT):
            raise ValueError(f"{name}: {_NAMES.get(status, 'error')} ({status})")
        raise ErvfError(name, status)
