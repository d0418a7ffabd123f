"""ctypes front end of ``oracle/_ref/libervf_ref.so`` -- the reference's own
CUDA kernels (built by ``oracle/build_ref.py``).

TEST INFRASTRUCTURE: used by tests/ to pin the CPU oracle and the product
against the reference implementation on a GPU, and to generate the golden
fixtures under tests/golden/.  Never imported by the product package.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libervf_ref.so"

_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_GEMV = [_vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _f, _vp]
SIGS = {
    "ref_gemv_rows": _GEMV,
    "ref_gemv_ervf16": _GEMV,
    "ref_gemv_ervf_w4": _GEMV,
    "ref_gemv_ervf_w8": _GEMV,
    "ref_gemv_ervf_w32": _GEMV,
    "ref_gemv_ervf_ind": [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _sz, _sz, _vp],
    "ref_weighted_accumulate": [_vp, _vp, _f, _vp, _i, _vp],
    "ref_down_masked": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _vp],
    "ref_route_topk": [_vp, _vp, _vp, _vp, _i, _i, _f, _i, _vp],
    "ref_cache_assign": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _vp],
    "ref_gemv_bf16": [_vp, _vp, _vp, _i, _i, _vp],
    "ref_gemv_f32": [_vp, _vp, _vp, _i, _i, _vp],
    "ref_panel_scan": [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp],
    "ref_gemm_rows_b": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp],
    "ref_down_masked_b": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _i, _i, _i, _i, _vp],
    "ref_reduce_partials_scatter": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "ref_reduce_slots": [_vp, _vp, _vp, _i, _i, _i, _vp],
}

_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(LIB_PATH))
        for n, a in SIGS.items():
            getattr(L, n).argtypes = a
            getattr(L, n).restype = ctypes.c_int
        _lib = L
    return _lib


def call(name, *args):
    st = getattr(lib(), name)(*args)
    if st != 0:
        raise RuntimeError(f"{name} failed ({st})")


def ervf_fn(width: int) -> str:
    return {4: "ref_gemv_ervf_w4", 8: "ref_gemv_ervf_w8", 16: "ref_gemv_ervf16",
            32: "ref_gemv_ervf_w32", 256: "ref_gemv_rows"}[width]
