"""ervf_moe_down_routesum_static: the routed sum with the library's own fixed
scratch array, called through the C ABI and compared bit for bit with
ervf_moe_down_routesum given a caller scratch buffer.  Named to run last, so
it also runs after every other GPU test has used the library."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, x_regime

pytestmark = pytest.mark.gpu

HIDDEN, INTER, N_EXPERTS = 2688, 1856, 8


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.fixture(scope="module")
def down_bank(cuda):
    dns = [random_nvfp4(HIDDEN, INTER, seed=2500 + e) for e in range(N_EXPERTS)]
    g = np.array([[d[2], 1.0] for d in dns], np.float32)
    return {
        "dns": dns,
        "c": _t(np.concatenate([d[0] for d in dns]), cuda),
        "s": _t(np.concatenate([d[1] for d in dns]), cuda),
        "g": _t(g, cuda),
    }


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _args(bank, ids, w, k, act, base, resid, out, hidden=HIDDEN):
    return (_p(bank["c"]), _p(bank["s"]), HIDDEN * INTER // 2, HIDDEN * INTER // 16, _p(ids),
            _p(bank["g"]), _p(w), k, _p(act), _p(base), _p(resid), _p(out), hidden, INTER)


def _routing(seed, k):
    r = np.random.default_rng(seed)
    ids = r.choice(N_EXPERTS, size=k, replace=False).astype(np.int32)
    w = r.uniform(0.05, 0.5, size=k).astype(np.float32)
    act = np.maximum(r.standard_normal(k * INTER), 0).astype(np.float32) ** 2
    return ids, w, act


def test_static_scratch_matches_caller_scratch_twice(cuda, oracle, down_bank):
    """Calls in a row on the fixed array.  With ERVF_LAUNCH_PDL, or one route
    slot, the route sum runs through the array's group counters; the
    unflagged 8-slot call takes the cluster route sum (no scratch)."""
    from ervf_b200 import _lib

    nbytes = _lib.load().ervf_routesum_scratch_bytes(HIDDEN, 8)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    pdl = _lib.LAUNCH_PDL
    cases = [(11, 6, "resid", pdl), (12, 8, "base", pdl), (13, 1, "resid", 0), (14, 8, "base", 0),
             (15, 3, "resid", pdl)]
    for seed, k, kind, flags in cases:  # calls in a row, different routings
        ids_h, w_h, act_h = _routing(seed, k)
        v = x_regime(HIDDEN, "random", seed=seed)
        ids, w, act, vv = _t(ids_h, cuda), _t(w_h, cuda), _t(act_h, cuda), _t(v, cuda)
        base, resid = (vv, None) if kind == "base" else (None, vv)
        want = torch.full((HIDDEN,), float("nan"), device=cuda)
        got = torch.full((HIDDEN,), float("nan"), device=cuda)
        _lib.call("ervf_moe_down_routesum", *_args(down_bank, ids, w, k, act, base, resid, want),
                  _p(scratch), ctypes.c_size_t(nbytes), 0, flags, _stream())
        _lib.call("ervf_moe_down_routesum_static",
                  *_args(down_bank, ids, w, k, act, base, resid, got), 0, flags, _stream())
        torch.cuda.synchronize()
        assert bits_equal(got.cpu().numpy(), want.cpu().numpy())
        # and against the oracle: route-order fmaf over the down GEMVs
        acc = v.copy() if kind == "base" else np.zeros(HIDDEN, np.float32)
        for s, e in enumerate(ids_h):
            dc, ds, dg = down_bank["dns"][e]
            y = oracle.nvfp4_gemv(dc, ds, act_h[s * INTER:(s + 1) * INTER], dg, HIDDEN, INTER)
            acc = oracle.weighted_accumulate(acc, y, w_h[s])
        if kind == "resid":
            acc = (v + acc).astype(np.float32)
        assert bits_equal(got.cpu().numpy(), acc)


def test_static_scratch_rejects_oversize(cuda, down_bank):
    from ervf_b200 import _lib

    ids_h, w_h, act_h = _routing(23, 8)
    ids, w, act = _t(ids_h, cuda), _t(w_h, cuda), _t(act_h, cuda)
    out = torch.zeros(HIDDEN, device=cuda)
    big_ids = _t(np.arange(9, dtype=np.int32) % N_EXPERTS, cuda)
    big_w = _t(np.full(9, 0.1, np.float32), cuda)
    big_act = torch.zeros(9 * INTER, device=cuda)
    with pytest.raises(ValueError, match="fixed scratch"):
        _lib.call("ervf_moe_down_routesum_static",
                  *_args(down_bank, big_ids, big_w, 9, big_act, None, None, out), 0, 0, _stream())
    with pytest.raises(ValueError, match="fixed scratch"):
        _lib.call("ervf_moe_down_routesum_static",
                  *_args(down_bank, ids, w, 8, act, None, None, out, hidden=8200), 0, 0, _stream())
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0  # nothing ran
