"""SweepMoE (the reference's expert-major block API, sweepspec.py:244-375)
against the reference's own SweepMoE kernels compiled from its source
(oracle/_ref/libervf_ref.so), bit for bit: gemm_into (gemm_nvfp4_rows_b),
down_union (panel_scan + gemm_down_masked_b over the union mask +
reduce_partials_scatter), reduce_slots, and a whole moe_block."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, x_regime

pytestmark = pytest.mark.gpu

HIDDEN, INTER = 2688, 1856


@pytest.fixture(scope="module")
def ref(cuda):
    import ref as r

    if not r.available():
        pytest.skip("oracle/_ref/libervf_ref.so not built (needs the reference tree at build time)")
    return r


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.fixture(scope="module")
def sweep(fused):
    from ervf_b200.sweep import SweepMoE

    return SweepMoE(fused, None)


@pytest.mark.parametrize("n,relu2", [(1, True), (5, False), (8, True)])
def test_gemm_into_equals_reference_batched_kernel(ref, fused, sweep, cuda, n, relu2):
    rows, cols = INTER, HIDDEN
    codes, scales, g = random_nvfp4(rows, cols, seed=40 + n, full_range=True)
    x_all = np.stack([x_regime(cols, "random", seed=s) for s in range(10)]).astype(np.float32)
    nodes = np.random.default_rng(n).integers(0, 10, n).astype(np.int32)  # repeats allowed
    c, s_, xd, nd = _t(codes, cuda), _t(scales, cuda), _t(x_all, cuda), _t(nodes, cuda)
    want = torch.full((n * rows,), float("nan"), device=cuda)
    ref.call("ref_gemm_rows_b", c.data_ptr(), s_.data_ptr(), fused.e2m1.data_ptr(), fused.e4m3.data_ptr(),
             xd.data_ptr(), nd.data_ptr(), want.data_ptr(), float(g), rows, cols, n, int(relu2), _s())
    got = torch.full((n * rows,), float("nan"), device=cuda)
    sweep.gemm_into(got, c, s_, xd, nd, g, rows, cols, n, apply_relu2=relu2)
    torch.cuda.synchronize()
    assert bits_equal(got.cpu().numpy(), want.cpu().numpy())


def _ref_down_union(ref, fused, cuda, bank_d, acts, dst, contrib, g, n, nchunks=8):
    """The reference's down_union sequence (gatherless) on its own kernels."""
    st = fused.alloc_masked_state(HIDDEN, INTER)
    act_sum = _t(acts[:n].sum(axis=0).astype(np.float32), cuda)
    acts_d = _t(acts, cuda)
    partials = torch.zeros(n * nchunks * HIDDEN, device=cuda)
    ref.call("ref_panel_scan", act_sum.data_ptr(), INTER, st["masks"].data_ptr(), st["plist"].data_ptr(),
             st["pcount"].data_ptr(), st["nz"].data_ptr(), st["nzc"].data_ptr(), _s())
    ref.call("ref_down_masked_b", bank_d.data_ptr(), acts_d.data_ptr(), st["plist"].data_ptr(),
             st["masks"].data_ptr(), st["pcount"].data_ptr(), fused.e2m1.data_ptr(), fused.e4m3.data_ptr(),
             partials.data_ptr(), float(g), HIDDEN, INTER, n, nchunks, _s())
    ref.call("ref_reduce_partials_scatter", partials.data_ptr(), dst.data_ptr(), contrib.data_ptr(),
             HIDDEN, nchunks, n, _s())
    torch.cuda.synchronize()


@pytest.mark.parametrize("n", [1, 3, 8])
def test_down_union_equals_reference(ref, fused, sweep, oracle, cuda, n):
    codes, scales, g = random_nvfp4(HIDDEN, INTER, seed=70 + n)
    bank_d = _t(oracle.panel_major(codes, scales, HIDDEN, INTER), cuda)
    r = np.random.default_rng(n)
    acts = np.maximum(r.standard_normal((n, INTER)), 0).astype(np.float32) ** 2  # ~50 % zeros
    acts[:, 100:300] = 0.0  # whole zero panels for every node
    for b in range(n):  # and a panel that only node b leaves empty: the union list differs
        acts[b, 16 * (30 + b):16 * (31 + b)] = 0.0
    top_k, B = 6, 8
    dst = _t(r.choice(B * top_k, n, replace=False).astype(np.int32), cuda)
    want = torch.zeros(B * top_k * HIDDEN, device=cuda)
    _ref_down_union(ref, fused, cuda, bank_d, acts, dst, want, g, n)
    state = sweep.alloc_state(HIDDEN, INTER, top_k, B)
    state["acts"][:n * INTER].copy_(_t(acts.reshape(-1), cuda))
    sweep.down_union(dst, bank_d.data_ptr(), state, g, HIDDEN, INTER, n)
    torch.cuda.synchronize()
    assert bits_equal(state["contrib"].cpu().numpy(), want.cpu().numpy())


def test_moe_block_equals_reference_sequence(ref, fused, sweep, oracle, cuda):
    """A whole layer for B = 4 nodes, top-6 over 8 experts: plan, gemm_into,
    down_union per expert, reduce_slots -- against the same sequence on the
    reference's kernels."""
    E, top_k, B = 8, 6, 4
    ups = [random_nvfp4(INTER, HIDDEN, seed=800 + e) for e in range(E)]
    dns = [random_nvfp4(HIDDEN, INTER, seed=900 + e) for e in range(E)]
    panels = np.concatenate([oracle.panel_major(d[0], d[1], HIDDEN, INTER) for d in dns])
    bank_d = _t(panels, cuda)
    globals_h = np.array([[d[2], u[2]] for u, d in zip(ups, dns)], np.float32)
    cache = {"map": np.arange(E), "codes": _t(np.concatenate([u[0] for u in ups]), cuda),
             "scales": _t(np.concatenate([u[1] for u in ups]), cuda)}
    rt = SimpleNamespace(hidden=HIDDEN, moe_inter=INTER, top_k=top_k,
                         bank=[{"globals": globals_h, "down_base_ptr": bank_d.data_ptr()}], cache=[cache])
    r = np.random.default_rng(3)
    routes = np.stack([r.choice(E, top_k, replace=False) for _ in range(B)]).astype(np.int32)
    weights = r.uniform(0.05, 0.3, (B, top_k)).astype(np.float32)
    x_all = np.stack([x_regime(HIDDEN, "bf16", seed=10 + b) for b in range(B)]).astype(np.float32)
    x_d = _t(x_all, cuda)
    groups = sweep.plan(routes, top_k)
    plan = sweep.compile_plan(groups, top_k)
    # ours
    state = sweep.alloc_state(HIDDEN, INTER, top_k, B)
    state["weights"].copy_(_t(weights.reshape(-1), cuda))
    out = x_d.clone()
    sweep.moe_block(out, rt, 0, x_d, plan, state, B)
    torch.cuda.synchronize()
    # the reference's kernels, in the reference's order
    contrib = torch.zeros(B * top_k * HIDDEN, device=cuda)
    acts = torch.zeros(B * INTER, device=cuda)
    up_code, up_scale = INTER * HIDDEN // 2, INTER * HIDDEN // 16
    pbytes = HIDDEN * INTER // 2 + HIDDEN * INTER // 16
    for e, nodes, dst, n in plan:
        ref.call("ref_gemm_rows_b", cache["codes"][e * up_code:].data_ptr(),
                 cache["scales"][e * up_scale:].data_ptr(), fused.e2m1.data_ptr(), fused.e4m3.data_ptr(),
                 x_d.data_ptr(), nodes.data_ptr(), acts.data_ptr(), float(globals_h[e, 1]), INTER, HIDDEN, n,
                 1, _s())
        torch.cuda.synchronize()
        a = acts[:n * INTER].cpu().numpy().reshape(n, INTER)
        _ref_down_union(ref, fused, cuda, bank_d[e * pbytes:], np.ascontiguousarray(a), dst, contrib,
                        globals_h[e, 0], n)
    want = x_d.clone()
    w_d = _t(weights.reshape(-1), cuda)
    ref.call("ref_reduce_slots", contrib.data_ptr(), w_d.data_ptr(), want.data_ptr(), HIDDEN, top_k, B, _s())
    torch.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), want.cpu().numpy())
