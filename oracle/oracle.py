"""numpy front end of the C oracle (``ervf_oracle.c``).

TEST INFRASTRUCTURE.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` import this module, and only to check or time against the
CUDA product.  The product package ``ervf_b200`` never imports it.

The C library is the bit-exact restatement of kennydd001/ervf's GEMV
arithmetic (file:line citations in ``ervf_oracle.c``).  Parity status: pinned
against the reference's codec known-answer tests
(``tests/lightningstream_nemotron/test_nvfp4.py:19-133``, re-hosted in
``tests/test_codec.py``) and against the reference's own CUDA kernels compiled
for sm_100a by ``oracle/build_ref.py`` and run on a B200
(``tests/test_ref_pin_gpu.py``, fixtures in ``tests/golden/``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
SRC_PATH = HERE / "ervf_oracle.c"

TREE_ERVF = 0
TREE_LEGACY = 1

_lib = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc (no fast-math, no FP contraction)."""
    if LIB_PATH.exists() and not force and LIB_PATH.stat().st_mtime >= SRC_PATH.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           "-std=c11", "-o", str(tmp), str(SRC_PATH), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SRC_PATH.stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oracle_luts.argtypes = [_f32p, _f32p, _f32p]
        L.oracle_nvfp4_gemv.argtypes = [_u8p, _u8p, _f32p, _f32p, ctypes.c_float,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_int]
        L.oracle_weighted_accumulate.argtypes = [_f32p, _f32p, ctypes.c_float, ctypes.c_int]
        L.oracle_expert.argtypes = [_u8p, _u8p, ctypes.c_float, _u8p, _u8p, ctypes.c_float,
                                    _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.oracle_panel_major.argtypes = [_u8p, _u8p, _u8p, ctypes.c_int, ctypes.c_int]
        L.oracle_down_masked.argtypes = [_u8p, _f32p, _f32p, ctypes.c_float, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int]
        L.oracle_bf16_gemv.argtypes = [_u16p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int]
        L.oracle_f32_gemv.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.oracle_route_topk.argtypes = [_f32p, _f32p, _i32p, _f32p, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_float, ctypes.c_int]
        L.oracle_cache_assign.argtypes = [_i32p] * 8 + [ctypes.c_int, ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def luts():
    """(e2m1 f32[16], e4m3 f32[256] with NaN->0, e4m3 raw f32[256] with NaN)."""
    e2m1 = np.zeros(16, np.float32)
    dev = np.zeros(256, np.float32)
    raw = np.zeros(256, np.float32)
    lib().oracle_luts(_p(e2m1, _f32p), _p(dev, _f32p), _p(raw, _f32p))
    return e2m1, dev, raw


def nvfp4_gemv(codes, scales, x, global_scale, rows, cols, apply_relu2=False,
               out_scale=1.0, tree=TREE_ERVF) -> np.ndarray:
    codes, scales, x = _u8(codes).reshape(-1), _u8(scales).reshape(-1), _f32(x).reshape(-1)
    if codes.size < rows * cols // 2 or scales.size < rows * cols // 16 or x.size < cols:
        raise ValueError("oracle: buffer smaller than rows x cols")
    out = np.zeros(rows, np.float32)
    lib().oracle_nvfp4_gemv(_p(codes, _u8p), _p(scales, _u8p), _p(x, _f32p), _p(out, _f32p),
                            np.float32(global_scale), rows, cols, int(bool(apply_relu2)),
                            np.float32(out_scale), tree)
    return out


def weighted_accumulate(dst, src, weight) -> np.ndarray:
    dst = _f32(dst).copy()
    src = _f32(src)
    lib().oracle_weighted_accumulate(_p(dst, _f32p), _p(src, _f32p), np.float32(weight),
                                     dst.size)
    return dst


def expert(up_c, up_s, up_g, dn_c, dn_s, dn_g, x, hidden, inter):
    """Returns (act f32[inter], out f32[hidden]) of FusedNVFP4.expert."""
    act = np.zeros(inter, np.float32)
    out = np.zeros(hidden, np.float32)
    up_c, up_s, dn_c, dn_s, x = _u8(up_c), _u8(up_s), _u8(dn_c), _u8(dn_s), _f32(x)
    lib().oracle_expert(_p(up_c, _u8p), _p(up_s, _u8p), np.float32(up_g),
                        _p(dn_c, _u8p), _p(dn_s, _u8p), np.float32(dn_g),
                        _p(x, _f32p), _p(act, _f32p), _p(out, _f32p), hidden, inter)
    return act, out


def moe_block(x, experts, ids, weights, hidden, inter, init=None):
    """Route-order sum of FusedNVFP4.expert outputs (runtime.py:588-596):
    out starts at ``init`` (zeros, or the shared-expert output) and takes
    out = fmaf(contrib_s, w_s, out) for s = 0..k-1 in ROUTE order."""
    out = np.zeros(hidden, np.float32) if init is None else _f32(init).copy()
    for s, e in enumerate(ids):
        up_c, up_s, up_g, dn_c, dn_s, dn_g = experts[int(e)]
        _, contrib = expert(up_c, up_s, up_g, dn_c, dn_s, dn_g, x, hidden, inter)
        out = weighted_accumulate(out, contrib, weights[s])
    return out


def panel_major(codes, scales, rows, inter) -> np.ndarray:
    npanel = inter // 16
    block = np.zeros(npanel * (rows + 16 * (rows // 2)), np.uint8)
    codes, scales = _u8(codes), _u8(scales)
    lib().oracle_panel_major(_p(codes, _u8p), _p(scales, _u8p), _p(block, _u8p), rows, inter)
    return block


def down_masked(bank, act, global_scale, rows, inter, nchunks=8) -> np.ndarray:
    out = np.zeros(rows, np.float32)
    bank, act = _u8(bank), _f32(act)
    lib().oracle_down_masked(_p(bank, _u8p), _p(act, _f32p), _p(out, _f32p),
                             np.float32(global_scale), rows, inter, nchunks)
    return out


def bf16_gemv(W_u16, x, rows, cols, batch=1) -> np.ndarray:
    W = np.ascontiguousarray(W_u16, dtype=np.uint16)
    x = _f32(x)
    out = np.zeros(batch * rows, np.float32)
    lib().oracle_bf16_gemv(_p(W, _u16p), _p(x, _f32p), _p(out, _f32p), rows, cols, batch)
    return out.reshape(batch, rows)


def f32_gemv(W, x, rows, cols) -> np.ndarray:
    """gemv_f32 (gpu_kernels.py:51-74) at the reference's 256-thread block."""
    W, x = _f32(W), _f32(x)
    out = np.zeros(rows, np.float32)
    lib().oracle_f32_gemv(_p(W, _f32p), _p(x, _f32p), _p(out, _f32p), rows, cols)
    return out


def route_topk(rlog, gate_b, top_k, scaling=1.0, bad_pick=0):
    rlog, gate_b = _f32(rlog), _f32(gate_b)
    n = rlog.size
    ids = np.zeros(top_k, np.int32)
    w = np.zeros(top_k, np.float32)
    lib().oracle_route_topk(_p(rlog, _f32p), _p(gate_b, _f32p), _p(ids, _i32p),
                            _p(w, _f32p), n, top_k, np.float32(scaling), bad_pick)
    return ids, w


def cache_assign(state: dict, ids, cap, top_k):
    """Mutates the int32 arrays of ``state`` (slot_of, expert_of, last_used,
    state2, stats2) in place; returns (slots, need)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    slots = np.zeros(top_k, np.int32)
    need = np.zeros(top_k, np.int32)
    lib().oracle_cache_assign(_p(state["slot_of"], _i32p), _p(state["expert_of"], _i32p),
                              _p(state["last_used"], _i32p), _p(state["state2"], _i32p),
                              _p(ids, _i32p), _p(slots, _i32p), _p(need, _i32p),
                              _p(state["stats2"], _i32p), cap, top_k)
    return slots, need


def dequant_f32(codes, scales, global_scale, rows, cols) -> np.ndarray:
    """FP32 dequantisation with the device tables (E4M3 NaN -> 0): the first
    half of the CPU dequant-then-matmul baseline (nvfp4.py:192-225 semantics,
    in fp32 as the kernels compute w = RN(e2m1 * RN(e4m3 * g)))."""
    e2m1, e4m3, _ = luts()
    codes = _u8(codes).reshape(rows, cols // 2)
    scales = _u8(scales).reshape(rows, cols // 16)
    nib = np.empty((rows, cols), np.uint8)
    nib[:, 0::2] = codes & 15
    nib[:, 1::2] = codes >> 4
    s = (e4m3[scales] * np.float32(global_scale)).astype(np.float32)
    return (e2m1[nib] * np.repeat(s, 16, axis=1)).astype(np.float32)
