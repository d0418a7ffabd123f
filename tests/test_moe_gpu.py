"""Routed-expert block on the GPU: the fused expert (up -> relu^2 -> down),
the route-order weighted sum, and the one-launch grouped forms, against the
CPU oracle bit for bit (config 1 shape: hidden 2688, inter 1856, top-6)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, rel_l2, x_regime

pytestmark = pytest.mark.gpu

HIDDEN, INTER = 2688, 1856


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.fixture(scope="module")
def bank(cuda):
    """8 experts, stacked like the resident bank: up row-major, down row-major."""
    n = 8
    ups = [random_nvfp4(INTER, HIDDEN, seed=1000 + e) for e in range(n)]
    dns = [random_nvfp4(HIDDEN, INTER, seed=1500 + e) for e in range(n)]
    globals_h = np.array([[d[2], u[2]] for u, d in zip(ups, dns)], np.float32)
    return {
        "ups": ups, "dns": dns, "globals": globals_h,
        "up_c": _t(np.concatenate([u[0] for u in ups]), cuda),
        "up_s": _t(np.concatenate([u[1] for u in ups]), cuda),
        "dn_c": _t(np.concatenate([d[0] for d in dns]), cuda),
        "dn_s": _t(np.concatenate([d[1] for d in dns]), cuda),
        "g_d": _t(globals_h, cuda),
    }


def test_expert_matches_oracle(fused, oracle, bank, cuda):
    x = x_regime(HIDDEN, "bf16", seed=1)
    for e in (0, 5):
        (uc, us, ug), (dc, ds, dg) = bank["ups"][e], bank["dns"][e]
        act = torch.zeros(INTER, device=cuda)
        out = torch.zeros(HIDDEN, device=cuda)
        fused.expert(_t(uc, cuda), _t(us, cuda), ug, _t(dc, cuda), _t(ds, cuda), dg, _t(x, cuda),
                     act, out, HIDDEN, INTER)
        torch.cuda.synchronize()
        want_act, want_out = oracle.expert(uc, us, ug, dc, ds, dg, x, HIDDEN, INTER)
        assert bits_equal(act.cpu().numpy(), want_act)
        assert bits_equal(out.cpu().numpy(), want_out)


def test_accumulate_route_order(fused, oracle, cuda):
    r = np.random.default_rng(3)
    dst = r.standard_normal(HIDDEN).astype(np.float32)
    d = _t(dst, cuda)
    want = dst
    for s in range(6):
        src = r.standard_normal(HIDDEN).astype(np.float32)
        w = np.float32(r.uniform(0.05, 0.4))
        fused.accumulate_into(d, _t(src, cuda), float(w), HIDDEN)
        want = oracle.weighted_accumulate(want, src, w)
    torch.cuda.synchronize()
    assert bits_equal(d.cpu().numpy(), want)


@pytest.mark.parametrize("width", [0, 16, 4])
def test_grouped_up_and_routesum_match_unfused(fused, oracle, bank, cuda, width):
    k = 6
    ids_h = np.array([3, 7, 0, 5, 1, 6], np.int32)
    rlog = np.random.default_rng(5).standard_normal(8).astype(np.float32)
    w_h = np.abs(rlog[:k]) / np.abs(rlog[:k]).sum()
    w_h = w_h.astype(np.float32)
    x = x_regime(HIDDEN, "bf16", seed=2)
    base = x_regime(HIDDEN, "random", seed=4)
    ids = _t(ids_h, cuda)
    w = _t(w_h, cuda)
    act = torch.zeros(k * INTER, device=cuda)
    out = torch.zeros(HIDDEN, device=cuda)
    fused.ervf_width = width
    fused.moe_up_grouped(bank["up_c"], bank["up_s"], INTER * HIDDEN // 2, INTER * HIDDEN // 16,
                         ids, bank["g_d"], k, _t(x, cuda), act, INTER, HIDDEN)
    fused.moe_down_routesum(bank["dn_c"], bank["dn_s"], HIDDEN * INTER // 2, HIDDEN * INTER // 16,
                            ids, bank["g_d"], w, k, act, out, HIDDEN, INTER, base=_t(base, cuda))
    fused.ervf_width = 0
    torch.cuda.synchronize()
    experts = {e: (*bank["ups"][e], *bank["dns"][e]) for e in range(8)}
    want = oracle.moe_block(x, experts, ids_h, w_h, HIDDEN, INTER, init=base)
    assert bits_equal(out.cpu().numpy(), want)
    # act slots are the unfused up GEMVs
    for s, e in enumerate(ids_h):
        uc, us, ug = bank["ups"][e]
        a = oracle.nvfp4_gemv(uc, us, x, ug, INTER, HIDDEN, apply_relu2=True)
        assert bits_equal(act[s * INTER:(s + 1) * INTER].cpu().numpy(), a)


def test_decoder_step_pdl_chain_matches_oracle(fused, oracle, bank, cuda):
    """Three layers of the decode step -- batched routing, then the
    PDL-chained per-layer launches with and without the L2 prefetch, eager
    and in a CUDA graph -- equal the oracle's route-order recurrence."""
    from ervf_b200.moe import ExpertBank, MoEDecoder

    L, E, k = 3, 8, 6
    eb = ExpertBank(L, E, HIDDEN, INTER, cuda)
    for l in range(L):
        for e in range(E):
            eb.upload_expert(l, e, bank["ups"][(e + l) % E], bank["dns"][(e + 2 * l) % E])
    dec = MoEDecoder(eb, k)
    r = np.random.default_rng(17)
    rl = r.standard_normal((L, E)).astype(np.float32)
    x = x_regime(HIDDEN, "bf16", seed=21)
    xd, rd = _t(x, cuda), _t(rl, cuda)
    for use_graph, prefetch in ((False, True), (True, True), (False, False), (True, False)):
        dec.prefetch = prefetch
        dec.xbuf.fill_(float("nan"))
        if use_graph:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                dec.step(xd, rd)
            torch.cuda.current_stream().wait_stream(s)
            with torch.cuda.graph(g):
                y = dec.step(xd, rd)
            g.replay()
        else:
            y = dec.step(xd, rd)
        torch.cuda.synchronize()
        want = x.copy()
        for l in range(L):
            ids, w = oracle.route_topk(rl[l], np.zeros(E, np.float32), k)
            experts = {e: (*bank["ups"][(e + l) % E], *bank["dns"][(e + 2 * l) % E]) for e in range(E)}
            want = (want + oracle.moe_block(want, experts, ids, w, HIDDEN, INTER)).astype(np.float32)
            assert np.array_equal(dec.ids[l].cpu().numpy(), ids)
        assert bits_equal(y.cpu().numpy(), want), (use_graph, prefetch)


@pytest.mark.parametrize("hidden,inter,E,k,L", [(2688, 1856, 8, 6, 3), (1024, 512, 8, 4, 2),
                                                 (4096, 2048, 4, 2, 2), (512, 1024, 6, 1, 3)])
def test_token_launch_equals_layer_chain(fused, cuda, hidden, inter, E, k, L):
    """ervf_moe_token (every layer of a token in one launch) equals the
    per-layer launches (ervf_moe_layer) bit for bit on the same routes, for
    three tokens back to back on one scratch, whose counters the kernel
    leaves zero."""
    from ervf_b200.moe import ExpertBank, MoEDecoder

    eb = ExpertBank.synthetic(L, E, hidden, inter, cuda, seed=5)
    dec = MoEDecoder(eb, k)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(9)
    for t in range(3):
        rl = torch.randn(L, E, generator=gen, device=cuda)
        x = torch.randn(hidden, generator=gen, device=cuda) * 0.05
        dec.token = True
        y_tok = dec.step(x, rl).clone()
        dec.token = False
        y_ref = dec.step(x, rl).clone()
        torch.cuda.synchronize()
        assert np.isfinite(y_ref.cpu().numpy()).all()
        assert bits_equal(y_tok.cpu().numpy(), y_ref.cpu().numpy()), f"token {t}"
    n_ctr = 32 * (2 + L + L * k) + L * ((hidden + 31) // 32)
    assert int(dec.tok_scratch[:4 * n_ctr].view(torch.int32).abs().sum()) == 0
    from ervf_b200 import _lib

    assert _lib.load().ervf_device_status() == 0


def test_decoder_step_with_router_matches_oracle(fused, oracle, bank, cuda):
    """Three layers with the router on the device between them (router GEMV +
    top-k, up, down + routed sum per layer, PDL-chained, eager and in a CUDA
    graph) equal the oracle's recurrence x <- x + moe(x) with
    ids, w = route_topk(gemv_f32(gate_w, x))."""
    from ervf_b200.moe import ExpertBank, MoEDecoder

    L, E, k = 3, 8, 6
    eb = ExpertBank(L, E, HIDDEN, INTER, cuda)
    for l in range(L):
        for e in range(E):
            eb.upload_expert(l, e, bank["ups"][(e + l) % E], bank["dns"][(e + 2 * l) % E])
    dec = MoEDecoder(eb, k)
    r = np.random.default_rng(23)
    gw = r.standard_normal((L, E, HIDDEN)).astype(np.float32) * 0.05
    gb = r.standard_normal((L, E)).astype(np.float32) * 0.1
    x = x_regime(HIDDEN, "bf16", seed=29)
    xd, gwd, gbd = _t(x, cuda), _t(gw, cuda), _t(gb, cuda)
    want = x.copy()
    for l in range(L):
        rlog = oracle.f32_gemv(gw[l], want, E, HIDDEN)
        oid, _ = oracle.route_topk(rlog, gb[l], k)
        # routing weights with CUDA expf (the standalone device router on the
        # oracle's logits), so that the expert sums compare bit for bit
        ids_d = torch.zeros(k, dtype=torch.int32, device=cuda)
        w_d = torch.zeros(k, device=cuda)
        fused.route_topk(_t(rlog, cuda), gbd[l], ids_d, w_d, E, k, 1.0)
        torch.cuda.synchronize()
        ids, w = ids_d.cpu().numpy(), w_d.cpu().numpy()
        assert np.array_equal(ids, oid)
        experts = {e: (*bank["ups"][(e + l) % E], *bank["dns"][(e + 2 * l) % E]) for e in range(E)}
        want = (want + oracle.moe_block(want, experts, ids, w, HIDDEN, INTER)).astype(np.float32)
    # one launch for every router and expert (token), or the per-layer launches
    for token, use_graph in ((True, False), (True, True), (False, False), (False, True)):
        dec.token = dec.token_router = token
        dec.xbuf.fill_(float("nan"))
        if use_graph:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                dec.step_with_router(xd, gwd, gbd)
            torch.cuda.current_stream().wait_stream(s)
            with torch.cuda.graph(g):
                y = dec.step_with_router(xd, gwd, gbd)
            g.replay()
        else:
            y = dec.step_with_router(xd, gwd, gbd)
        torch.cuda.synchronize()
        assert bits_equal(y.cpu().numpy(), want), (token, use_graph)


@pytest.mark.parametrize("E,with_bias", [(128, True), (256, False), (44, True)])
def test_token_router_equals_layer_router(fused, cuda, E, with_bias):
    """The routed token launch (router items inside ervf_moe_token_router)
    gives the same ids, weights and output bits as the per-layer router +
    expert launches, for three tokens back to back."""
    from ervf_b200.moe import ExpertBank, MoEDecoder

    L, k = 3, 6
    eb = ExpertBank.synthetic(L, E, HIDDEN, INTER, cuda, seed=11)
    dec = MoEDecoder(eb, k, scaling=2.5)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(31)
    gw = torch.randn(L, E, HIDDEN, generator=gen, device=cuda) * 0.05
    gb = torch.randn(L, E, generator=gen, device=cuda) * 0.1 if with_bias else None
    for t in range(3):
        x = torch.randn(HIDDEN, generator=gen, device=cuda) * 0.05
        dec.token = dec.token_router = True
        y_tok = dec.step_with_router(x, gw, gb).clone()
        ids_tok, w_tok = dec.ids.clone(), dec.w.clone()
        dec.token = dec.token_router = False
        y_ref = dec.step_with_router(x, gw, gb).clone()
        torch.cuda.synchronize()
        assert torch.equal(ids_tok, dec.ids), t
        assert bits_equal(w_tok.cpu().numpy(), dec.w.cpu().numpy()), t
        assert np.isfinite(y_ref.cpu().numpy()).all()
        assert bits_equal(y_tok.cpu().numpy(), y_ref.cpu().numpy()), t
    from ervf_b200 import _lib

    assert _lib.load().ervf_device_status() == 0


def test_routesum_residual_matches_f64(fused, oracle, bank, cuda):
    """x + moe(x) against a float64 dequant reference (tolerance, not bits)."""
    from ervf_b200.formats import dequantize

    k = 6
    ids_h = np.array([2, 4, 6, 1, 0, 3], np.int32)
    w_h = np.full(k, 1.0 / k, np.float32)
    x = x_regime(HIDDEN, "bf16", seed=7)
    act = torch.zeros(k * INTER, device=cuda)
    out = torch.zeros(HIDDEN, device=cuda)
    xd = _t(x, cuda)
    fused.moe_up_grouped(bank["up_c"], bank["up_s"], INTER * HIDDEN // 2, INTER * HIDDEN // 16,
                         _t(ids_h, cuda), bank["g_d"], k, xd, act, INTER, HIDDEN)
    fused.moe_down_routesum(bank["dn_c"], bank["dn_s"], HIDDEN * INTER // 2, HIDDEN * INTER // 16,
                            _t(ids_h, cuda), bank["g_d"], _t(w_h, cuda), k, act, out, HIDDEN, INTER,
                            resid=xd)
    torch.cuda.synchronize()
    ref = x.astype(np.float64).copy()
    for s, e in enumerate(ids_h):
        uc, us, ug = bank["ups"][e]
        dc, ds, dg = bank["dns"][e]
        h = dequantize(uc, us, ug, INTER, HIDDEN) @ x.astype(np.float64)
        a = np.maximum(h, 0) ** 2
        ref += float(w_h[s]) * (dequantize(dc, ds, dg, HIDDEN, INTER) @ a)
    assert rel_l2(out.cpu().numpy(), ref) < 1e-5


def test_batched_step_matches_f64(fused, oracle, bank, cuda):
    """Expert-major batched decode (tensor-core path) of 8 tokens through two
    layers against float64 dequantise-then-matmul with the same routing."""
    from ervf_b200.formats import dequantize
    from ervf_b200.moe import ExpertBank, MoEDecoder

    L, E, k, T = 2, 8, 6, 8
    eb = ExpertBank(L, E, HIDDEN, INTER, cuda)
    for l in range(L):
        for e in range(E):
            eb.upload_expert(l, e, bank["ups"][(e + l) % E], bank["dns"][(e + 3 * l) % E])
    dec = MoEDecoder(eb, k)
    r = np.random.default_rng(23)
    rl = r.standard_normal((L, T, E)).astype(np.float32)
    x = np.stack([x_regime(HIDDEN, "bf16", seed=40 + t) for t in range(T)]).astype(np.float32)
    y = dec.step_batch(_t(x, cuda), _t(rl, cuda))
    torch.cuda.synchronize()
    ids = dec.bids.cpu().numpy().reshape(L, T, k)
    w = dec.bw.cpu().numpy().reshape(L, T, k)
    want = x.astype(np.float64)
    for l in range(L):
        nxt = want.copy()
        for t in range(T):
            oid, _ = oracle.route_topk(rl[l, t], np.zeros(E, np.float32), k)
            assert np.array_equal(ids[l, t], oid)
            for s in range(k):
                e = ids[l, t, s]
                uc, us, ug = bank["ups"][(e + l) % E]
                dc, ds, dg = bank["dns"][(e + 3 * l) % E]
                h = dequantize(uc, us, ug, INTER, HIDDEN) @ want[t]
                a = np.maximum(h, 0) ** 2
                nxt[t] += float(w[l, t, s]) * (dequantize(dc, ds, dg, HIDDEN, INTER) @ a)
        want = nxt
    # weights are exact in f16; activations after the first layer (and act)
    # are rounded to f16 (2^-12 relative), which is the ~4e-4 seen here
    y1 = y.cpu().numpy()
    assert rel_l2(y1, want) <= 1e-3
    # the K-split re-associates fp32 partial sums; a value that then rounds to
    # the other f16 neighbour as the next MMA operand moves by an f16 ulp
    # (2^-11 relative), so the two agree to the tolerance of this path
    dec.batch_ksplit = 2
    y2 = dec.step_batch(_t(x, cuda), _t(rl, cuda)).cpu().numpy()
    assert rel_l2(y2, want) <= 1e-3
    assert rel_l2(y2, y1) <= 1e-3


def test_moe_layer_entry_matches_oracle(oracle, bank, cuda):
    """ervf_moe_layer (up + down + route-order sum + residual, with and without
    the L2 prefetch of the next layer's records, with and without PDL) equals
    the oracle's routed block plus x, bit for bit."""
    from ervf_b200 import _lib
    from ervf_b200.fused_nvfp4 import ptr

    k = 6
    ids_h = np.array([2, 5, 7, 0, 3, 1], np.int32)
    nxt_h = np.array([4, 6, 1, 0, 7, 2], np.int32)
    w_h = np.random.default_rng(8).uniform(0.05, 0.4, k).astype(np.float32)
    x = x_regime(HIDDEN, "bf16", seed=12)
    ids, nxt, w, xd = _t(ids_h, cuda), _t(nxt_h, cuda), _t(w_h, cuda), _t(x, cuda)
    act = torch.zeros(k * INTER, device=cuda)
    nb = _lib.load().ervf_routesum_scratch_bytes(HIDDEN, k)
    scratch = torch.zeros(nb, dtype=torch.uint8, device=cuda)
    experts = {e: (*bank["ups"][e], *bank["dns"][e]) for e in range(8)}
    want = (x + oracle.moe_block(x, experts, ids_h, w_h, HIDDEN, INTER)).astype(np.float32)
    cb, sb = INTER * HIDDEN // 2, INTER * HIDDEN // 16
    for flags in (0, _lib.LAUNCH_PDL, _lib.LAUNCH_PDL | _lib.LAUNCH_IDS_READY):
        for pf in ((ptr(bank["up_c"]), ptr(bank["up_s"]), ptr(nxt)), (0, 0, 0)):
            out = torch.full((HIDDEN,), float("nan"), device=cuda)
            _lib.call("ervf_moe_layer", ptr(bank["up_c"]), ptr(bank["up_s"]), cb, sb, ptr(bank["dn_c"]),
                      ptr(bank["dn_s"]), cb, sb, ptr(ids), ptr(bank["g_d"]), ptr(w), k, ptr(xd),
                      ptr(act), ptr(out), HIDDEN, INTER, 8, ptr(scratch), nb, *pf, flags,
                      torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            assert bits_equal(out.cpu().numpy(), want), (flags, pf[2] != 0)
    # the scratch is left ready: every 32-row group counter (at its start) back at zero
    cnt = scratch[:HIDDEN * 4].view(torch.int32)[:(HIDDEN + 31) // 32]
    assert torch.count_nonzero(cnt).item() == 0
