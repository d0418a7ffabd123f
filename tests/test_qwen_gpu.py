"""Config 2: Qwen3-30B-A3B-shaped SwiGLU experts (hidden 2048, moe
intermediate 768, top-8 softmax routing) on the B200 schedule.

The reference's NVFP4 kernels have no SwiGLU epilogue and no softmax router,
so the GEMV products are checked bit for bit against the oracle, and the
SwiGLU / softmax arithmetic (which calls expf) against float32 numpy with a
tolerance; the whole block against a float64 dequantise-then-matmul."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, rel_l2, x_regime

pytestmark = pytest.mark.gpu

HIDDEN, INTER, E, K = 2048, 768, 16, 8


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _silu(v):
    v = v.astype(np.float32)
    return (v / (np.float32(1) + np.exp(-v))).astype(np.float32)


@pytest.fixture(scope="module")
def qbank(cuda):
    """16 experts: gate+up [2*768 x 2048] with gate / up rows interleaved
    (row 2i = gate i, row 2i+1 = up i), down [2048 x 768]."""
    ups = [random_nvfp4(2 * INTER, HIDDEN, seed=3000 + e) for e in range(E)]
    dns = [random_nvfp4(HIDDEN, INTER, seed=3500 + e) for e in range(E)]
    g = np.array([[d[2], u[2]] for u, d in zip(ups, dns)], np.float32)
    return {"ups": ups, "dns": dns, "globals": g,
            "up_c": _t(np.concatenate([u[0] for u in ups]), cuda),
            "up_s": _t(np.concatenate([u[1] for u in ups]), cuda),
            "dn_c": _t(np.concatenate([d[0] for d in dns]), cuda),
            "dn_s": _t(np.concatenate([d[1] for d in dns]), cuda),
            "g": _t(g, cuda)}


def _softmax_topk(rl, k):
    order = sorted(range(len(rl)), key=lambda e: (-float(rl[e]), e))[:k]
    top = np.float32(rl[order[0]])
    e = np.array([np.exp(np.float32(rl[i]) - top) for i in order], np.float32)
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    return np.array(order, np.int32), (e / s).astype(np.float32)


def test_softmax_router_matches_numpy(fused, cuda):
    r = np.random.default_rng(41)
    for layers, n, k in ((24, 128, 8), (3, 64, 4), (2, 300, 8)):
        rl = r.standard_normal((layers, n)).astype(np.float32)
        rl[0, 5] = rl[0, 9] = rl[0].max() + 1  # a tie: lower index first
        ids = torch.zeros(layers, k, dtype=torch.int32, device=cuda)
        w = torch.zeros(layers, k, device=cuda)
        fused.route_topk_softmax(_t(rl, cuda), ids, w, layers, n, k)
        torch.cuda.synchronize()
        for l in range(layers):
            oid, ow = _softmax_topk(rl[l], k)
            assert np.array_equal(ids[l].cpu().numpy(), oid)
            np.testing.assert_allclose(w[l].cpu().numpy(), ow, rtol=2e-6)
        assert ids[0, 0].item() == 5 and ids[0, 1].item() == 9


def test_swiglu_grouped_up_matches_oracle_products(fused, oracle, qbank, cuda):
    from ervf_b200 import _lib

    ids_h = np.array([3, 14, 0, 7, 9, 1, 12, 5], np.int32)
    x = x_regime(HIDDEN, "bf16", seed=8)
    act = torch.full((K * INTER,), float("nan"), device=cuda)
    fused.moe_up_grouped(qbank["up_c"], qbank["up_s"], 2 * INTER * HIDDEN // 2,
                         2 * INTER * HIDDEN // 16, _t(ids_h, cuda), qbank["g"], K, _t(x, cuda), act,
                         INTER, HIDDEN, flags=_lib.UP_SWIGLU)
    torch.cuda.synchronize()
    got = act.cpu().numpy().reshape(K, INTER)
    for s, e in enumerate(ids_h):
        uc, us, ug = qbank["ups"][e]
        y = oracle.nvfp4_gemv(uc, us, x, ug, 2 * INTER, HIDDEN)  # bit-exact products
        want = (_silu(y[0::2]) * y[1::2]).astype(np.float32)
        np.testing.assert_allclose(got[s], want, rtol=1e-6, atol=1e-30)


def test_swiglu_needs_b200_schedule(fused, qbank, cuda):
    from ervf_b200 import _lib

    act = torch.zeros(K * INTER, device=cuda)
    fused.ervf_width = 16
    try:
        with pytest.raises(ValueError):
            fused.moe_up_grouped(qbank["up_c"], qbank["up_s"], 2 * INTER * HIDDEN // 2,
                                 2 * INTER * HIDDEN // 16, _t(np.arange(K, dtype=np.int32), cuda),
                                 qbank["g"], K, torch.zeros(HIDDEN, device=cuda), act, INTER, HIDDEN,
                                 flags=_lib.UP_SWIGLU)
    finally:
        fused.ervf_width = 0


def test_qwen_block_matches_f64(fused, qbank, cuda):
    """softmax top-8 -> grouped gate+up SwiGLU -> down + route-order sum +
    residual, against a float64 dequantise-then-matmul of the same bytes."""
    from ervf_b200 import _lib
    from ervf_b200.formats import dequantize

    r = np.random.default_rng(5)
    rl = r.standard_normal((1, E)).astype(np.float32)
    x = x_regime(HIDDEN, "bf16", seed=9)
    ids = torch.zeros(1, K, dtype=torch.int32, device=cuda)
    w = torch.zeros(1, K, device=cuda)
    xd = _t(x, cuda)
    act = torch.zeros(K * INTER, device=cuda)
    out = torch.zeros(HIDDEN, device=cuda)
    fused.route_topk_softmax(_t(rl, cuda), ids, w, 1, E, K)
    fused.moe_up_grouped(qbank["up_c"], qbank["up_s"], 2 * INTER * HIDDEN // 2,
                         2 * INTER * HIDDEN // 16, ids[0], qbank["g"], K, xd, act, INTER, HIDDEN,
                         flags=_lib.UP_SWIGLU)
    fused.moe_down_routesum(qbank["dn_c"], qbank["dn_s"], HIDDEN * INTER // 2, HIDDEN * INTER // 16,
                            ids[0], qbank["g"], w[0], K, act, out, HIDDEN, INTER, resid=xd)
    torch.cuda.synchronize()
    ids_h, w_h = ids[0].cpu().numpy(), w[0].cpu().numpy()
    ref = x.astype(np.float64).copy()
    for s, e in enumerate(ids_h):
        uc, us, ug = qbank["ups"][e]
        dc, ds, dg = qbank["dns"][e]
        gu = dequantize(uc, us, ug, 2 * INTER, HIDDEN) @ x.astype(np.float64)
        gate, up = gu[0::2], gu[1::2]
        a = gate / (1.0 + np.exp(-gate)) * up
        ref += float(w_h[s]) * (dequantize(dc, ds, dg, HIDDEN, INTER) @ a)
    assert rel_l2(out.cpu().numpy(), ref) < 1e-5


def test_qwen_block_batch16_on_tensor_cores_matches_f64(fused, qbank, cuda):
    """Config 2 at batch 16: softmax top-8 routing, then the expert-major
    batched block on the tensor cores with the SwiGLU epilogue (gate / up row
    pairs), route-order sum and residual -- within rel-L2 1e-3 of a float64
    dequantise-then-matmul of the same bytes and routing (K-split 1 and 2)."""
    from ervf_b200.formats import dequantize

    T = 16
    r = np.random.default_rng(77)
    rl = r.standard_normal((T, E)).astype(np.float32)
    x = np.stack([x_regime(HIDDEN, "bf16", seed=60 + t) for t in range(T)]).astype(np.float32)
    ids = torch.zeros(T, K, dtype=torch.int32, device=cuda)
    w = torch.zeros(T, K, device=cuda)
    fused.route_topk_softmax(_t(rl, cuda), ids, w, T, E, K)
    ids_h, w_h = ids.cpu().numpy(), w.cpu().numpy()
    deq_up = {e: dequantize(*qbank["ups"][e][:2], qbank["ups"][e][2], 2 * INTER, HIDDEN) for e in range(E)}
    deq_dn = {e: dequantize(*qbank["dns"][e][:2], qbank["dns"][e][2], HIDDEN, INTER) for e in range(E)}
    ref = x.astype(np.float64).copy()
    for t in range(T):
        for s in range(K):
            e = int(ids_h[t, s])
            gu = deq_up[e] @ x[t].astype(np.float64)
            gate, up = gu[0::2], gu[1::2]
            ref[t] += float(w_h[t, s]) * (deq_dn[e] @ (gate / (1.0 + np.exp(-gate)) * up))
    for ksplit in (1, 2):
        out = torch.full((T, HIDDEN), float("nan"), device=cuda)
        fused.moe_batched(qbank["up_c"], qbank["up_s"], 2 * INTER * HIDDEN // 2, 2 * INTER * HIDDEN // 16,
                          qbank["dn_c"], qbank["dn_s"], HIDDEN * INTER // 2, HIDDEN * INTER // 16,
                          qbank["g"], ids, w, T, K, E, _t(x, cuda), out, HIDDEN, INTER, ksplit=ksplit,
                          swiglu=True)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, ref) <= 1e-3, (ksplit, rel_l2(got, ref))
