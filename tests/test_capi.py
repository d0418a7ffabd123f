"""The C-ABI library without a GPU: it loads, exports every entry point that
include/ervf_b200.h declares (and ctypes knows them all), and rejects bad
arguments before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ervf_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "ervf_b200.h"


def declared():
    return re.findall(r"^ERVF_API (?:int|size_t) (ervf_\w+)\(", HEADER.read_text(), flags=re.M)


def test_header_declares_entry_points():
    names = declared()
    assert len(names) >= 18 and len(set(names)) == len(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name


def test_binding_covers_header_exactly():
    assert set(declared()) == set(_lib.SIGNATURES)


def test_version():
    assert _lib.load().ervf_version() == 100


def test_null_and_shape_checks_need_no_device():
    lib = _lib.load()
    assert lib.ervf_nvfp4_gemv(None, None, None, None, 1.0, 8, 16, 0, 1.0, 0, 0, None) == _lib.ERR_NULL
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    # cols % 16 != 0 is rejected before any CUDA call
    assert lib.ervf_nvfp4_gemv(p, p, p, p, 1.0, 8, 24, 0, 1.0, 0, 0, None) == _lib.ERR_SHAPE
    assert lib.ervf_nvfp4_gemv(p, p, p, p, 1.0, 0, 16, 0, 1.0, 0, 0, None) == _lib.ERR_SHAPE
    assert lib.ervf_bf16_gemv(p, p, p, 4, 12, 1, None) == _lib.ERR_SHAPE
    assert lib.ervf_bf16_gemv(p, p, p, 4, 16, 9, None) == _lib.ERR_ARG
    assert lib.ervf_route_topk(p, p, p, p, 2000, 6, 1.0, 0, None) == _lib.ERR_SHAPE
    assert lib.ervf_weighted_accumulate(None, p, 1.0, 4, None) == _lib.ERR_NULL
    assert lib.ervf_down_masked(p, p, p, p, p, p, p, p, 1.0, 2688, 1856, 0, None) == _lib.ERR_ARG


def test_python_shim_raises_value_error():
    with pytest.raises(ValueError):
        _lib.call("ervf_nvfp4_gemv", None, None, None, None, 1.0, 8, 16, 0, 1.0, 0, 0, None)


def test_token_entries_check_arguments_without_a_device():
    lib = _lib.load()
    nb = lib.ervf_moe_token_scratch_bytes(24, 2688, 1856, 6)
    assert nb > 0 and lib.ervf_moe_token_scratch_bytes(0, 2688, 1856, 6) == 0
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    args = (p, 24, 2688 * 1856 // 2, 2688 * 1856 // 16, 2688 * 1856 // 2, 2688 * 1856 // 16, p, p, 6, 128,
            p, p, 2688, 1856, p)
    assert lib.ervf_moe_token(None, *args[1:], nb, 0, None) == _lib.ERR_NULL
    bad_shape = list(args)
    bad_shape[12] = 100  # hidden not a multiple of 32
    assert lib.ervf_moe_token(*bad_shape, nb, 0, None) == _lib.ERR_SHAPE
    assert lib.ervf_moe_token(*args, nb - 1, 0, None) == _lib.ERR_ARG  # scratch too small
    assert lib.ervf_moe_token(*args, nb, 0x40, None) == _lib.ERR_ARG   # unknown flag
    r = (p, 24, 2688 * 1856 // 2, 2688 * 1856 // 16, 2688 * 1856 // 2, 2688 * 1856 // 16, p, p, 6)
    tail = (p, p, 2688, 1856, p, nb, 0, None)
    assert lib.ervf_moe_token_router(*r, 512, 1.0, 0, *tail) == _lib.ERR_SHAPE   # > 256 experts
    assert lib.ervf_moe_token_router(*r, 128, 1.0, 2, *tail) == _lib.ERR_ARG     # bad_pick
    assert lib.ervf_moe_token_router(*r, 4, 1.0, 0, *tail) == _lib.ERR_SHAPE     # top_k > experts


def test_token_ep_entry_checks_arguments_without_a_device():
    """ervf_moe_token_ep rejects bad rank counts, peer tables and sizes before
    any CUDA call (the launch itself needs two or more GPUs)."""
    lib = _lib.load()
    nb = lib.ervf_moe_token_ep_scratch_bytes(24, 2688, 1856, 6)
    assert nb > 0
    assert lib.ervf_moe_token_ep_scratch_bytes(24, 2688, 1856, 0) == 0
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    peers = (ctypes.c_uint64 * 2)(0x10000, 0x20000)
    pp = ctypes.cast(peers, ctypes.c_void_p)
    head = (p, 24, 2688 * 1856 // 2, 2688 * 1856 // 16, 2688 * 1856 // 2, 2688 * 1856 // 16, p, p, 6, 128,
            p, p, 2688, 1856)

    def call(peer=pp, ranks=2, rank=0, nbytes=nb, timeout=5000, flags=0, hd=head):
        return lib.ervf_moe_token_ep(*hd, peer, ranks, rank, nbytes, timeout, flags, None)

    assert call(peer=None) == _lib.ERR_NULL
    assert call(ranks=1) == _lib.ERR_ARG      # one rank: ervf_moe_token
    assert call(ranks=9) == _lib.ERR_ARG      # at most 8 ranks
    assert call(rank=2) == _lib.ERR_ARG       # rank outside the group
    assert call(timeout=0) == _lib.ERR_ARG
    assert call(flags=0x40) == _lib.ERR_ARG   # unknown flag
    assert call(nbytes=nb - 1) == _lib.ERR_ARG  # scratch too small
    bad = list(head)
    bad[12] = 100                             # hidden not a multiple of 32
    assert call(hd=tuple(bad)) == _lib.ERR_SHAPE
    zero = (ctypes.c_uint64 * 2)(0x10000, 0)
    assert call(peer=ctypes.cast(zero, ctypes.c_void_p)) == _lib.ERR_NULL
    odd = (ctypes.c_uint64 * 2)(0x10000, 0x20010)
    assert call(peer=ctypes.cast(odd, ctypes.c_void_p)) == _lib.ERR_ALIGN


def test_token_ep_prepare_checks_arguments_without_a_device():
    lib = _lib.load()
    nb = lib.ervf_moe_token_ep_scratch_bytes(24, 2688, 1856, 6)
    assert lib.ervf_moe_token_ep_prepare(None, nb, 24, 2688, 1856, 6, None) == _lib.ERR_NULL
    assert lib.ervf_moe_token_ep_prepare(0x10000, nb, 0, 2688, 1856, 6, None) == _lib.ERR_SHAPE
    assert lib.ervf_moe_token_ep_prepare(0x10000, nb - 1, 24, 2688, 1856, 6, None) == _lib.ERR_ARG
    assert lib.ervf_moe_token_ep_prepare(0x10010, nb, 24, 2688, 1856, 6, None) == _lib.ERR_ALIGN
