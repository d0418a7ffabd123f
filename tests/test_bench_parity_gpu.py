"""Parity on exactly what bench.py times: the seeded
24-layer x 128-expert bank that bench.py builds, decode tokens at batch 1
through the PDL-chained, L2-prefetching decode step (eager and the captured
graph), bit for bit against the C oracle; and the batch-32 expert-major
tensor-core block over all 24 layers (K-split 1 and 2) within rel-L2 1e-3 of
a float64 dequantise-then-matmul recurrence.

The recurrence x_{l+1} = x_l + moe_l(x_l) has no normalisation and relu^2 is
quadratic, so from bench.py's N(0, 1) hidden states it overflows to inf (and
then NaN) after about a dozen layers -- the bytes streamed and the work done
per layer do not depend on the values.  The benched token is therefore
checked layer by layer (each layer of the product against the oracle's same
layer on the product's own input, NaN positions compared as NaN), and a token
scaled by 1/16, whose recurrence stays finite through all 24 layers, through
the whole captured graph."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits_equal, dequant_torch, rel_l2

pytestmark = pytest.mark.gpu

HIDDEN, INTER, N_EXPERTS, TOP_K, N_LAYERS = 2688, 1856, 128, 6, 24


@pytest.fixture(scope="module")
def bench_bank(cuda):
    from ervf_b200.moe import ExpertBank

    bank = ExpertBank.synthetic(N_LAYERS, N_EXPERTS, HIDDEN, INTER, cuda)
    yield bank
    del bank
    torch.cuda.empty_cache()


def _bench_inputs(cuda, tokens):
    """bench.py's per-token router logits and bf16-valued hidden states."""
    g = torch.Generator(device=cuda)
    g.manual_seed(2)
    rlogs = torch.randn(tokens, N_LAYERS, N_EXPERTS, generator=g, device=cuda)
    xs = torch.randn(tokens, HIDDEN, generator=g, device=cuda)
    xs = (xs.view(torch.int32) & -65536).view(torch.float32)
    return rlogs, xs


def _same_bits_or_nan(a, b) -> bool:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and bits_equal(a[~na], b[~nb]))


def _oracle_layer(bank, oracle, cache, l, x, ids, w):
    experts = {}
    for e in ids:
        key = (l, int(e))
        if key not in cache:
            (uc, us, ug), (dc, ds, dg) = bank.expert_host(l, int(e))
            cache[key] = (uc, us, ug, dc, ds, dg)
        experts[int(e)] = cache[key]
    with np.errstate(all="ignore"):
        return (x + oracle.moe_block(x, experts, ids, w, HIDDEN, INTER)).astype(np.float32)


def _capture(dec, x_buf, r_buf, cuda):
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        dec.step(x_buf, r_buf)
    torch.cuda.current_stream(cuda).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = dec.step(x_buf, r_buf)
    return graph, y


def test_config4_benched_token_layer_by_layer(bench_bank, oracle, cuda):
    """bench.py's first timed token: routing of all 24 layers equal to the
    oracle's, every layer of the PDL chain (launched as the decode step
    launches it) equal to the oracle's layer on the same input, and the
    captured graph's output equal to the eager chain's."""
    from ervf_b200.moe import MoEDecoder

    dec = MoEDecoder(bench_bank, TOP_K)
    rlogs, xs = _bench_inputs(cuda, 6)
    t = 5  # bench.py's first timed token after 5 warm-up tokens
    x_buf = xs[t].clone()
    r_buf = rlogs[t].clone()
    dec.route(r_buf)
    torch.cuda.synchronize(cuda)
    rl = r_buf.cpu().numpy()
    ids_dev, w_dev = dec.ids.cpu().numpy(), dec.w.cpu().numpy()
    for l in range(N_LAYERS):
        ids, w = oracle.route_topk(rl[l], np.zeros(N_EXPERTS, np.float32), TOP_K)
        assert np.array_equal(ids_dev[l], ids), l
        np.testing.assert_allclose(w_dev[l], w, rtol=3e-7, atol=0)
    cache = {}
    cur = x_buf
    finite_layers = 0
    for l in range(N_LAYERS):
        nxt = torch.empty_like(cur)
        dec.layer(l, cur, nxt, first=(l == 0))
        torch.cuda.synchronize(cuda)
        xin = cur.cpu().numpy()
        want = _oracle_layer(bench_bank, oracle, cache, l, xin, ids_dev[l], w_dev[l])
        got = nxt.cpu().numpy()
        assert _same_bits_or_nan(got, want), f"layer {l}"
        finite_layers += int(np.isfinite(got).all())
        cur = nxt
    assert finite_layers >= 8  # the first layers carry finite values
    eager = cur.cpu().numpy()
    x_in = torch.zeros(HIDDEN, device=cuda)
    graph, y = _capture(dec, x_in, r_buf, cuda)
    x_in.copy_(xs[t])
    graph.replay()
    torch.cuda.synchronize(cuda)
    assert _same_bits_or_nan(y.cpu().numpy(), eager)
    del graph


def test_config4_finite_token_whole_graph_bit_exact(bench_bank, oracle, cuda):
    """Two tokens (bench.py's inputs scaled by 1/16: finite through every
    layer) through the captured 24-layer graph, replayed back to back, bit for
    bit against the oracle's recurrence."""
    from ervf_b200.moe import MoEDecoder

    dec = MoEDecoder(bench_bank, TOP_K)
    rlogs, xs = _bench_inputs(cuda, 2)
    xs = xs * (1.0 / 16.0)
    x_buf = torch.zeros(HIDDEN, device=cuda)
    r_buf = torch.zeros(N_LAYERS, N_EXPERTS, device=cuda)
    graph, y = _capture(dec, x_buf, r_buf, cuda)
    cache = {}
    for t in range(2):  # the scratch counters carry over between replays
        x_buf.copy_(xs[t])
        r_buf.copy_(rlogs[t])
        graph.replay()
        torch.cuda.synchronize(cuda)
        got = y.cpu().numpy()
        want = xs[t].cpu().numpy()
        ids_dev, w_dev = dec.ids.cpu().numpy(), dec.w.cpu().numpy()
        for l in range(N_LAYERS):
            want = _oracle_layer(bench_bank, oracle, cache, l, want, ids_dev[l], w_dev[l])
        assert np.isfinite(want).all()
        assert bits_equal(got, want), f"token {t}: max |d| {np.abs(got - want).max():.3e}"
    del graph


def _float64_batch_recurrence(bank, x0, ids, w):
    """x_{l+1} = x_l + sum_s w_s down_e(relu(up_e(x_l))^2) in float64 on the
    GPU, the experts dequantised from the bank's bytes."""
    T = x0.shape[0]
    x = x0.to(torch.float64)
    L = bank.n_layers
    for l in range(L):
        idl, wl = ids[l], w[l].to(torch.float64)
        nxt = x.clone()
        for e in torch.unique(idl).tolist():
            (uc, us, ug), (dc, ds, dg) = _expert_dev(bank, l, e)
            up = dequant_torch(uc, us, ug, INTER, HIDDEN)
            dn = dequant_torch(dc, ds, dg, HIDDEN, INTER)
            tok, slot = torch.nonzero(idl == e, as_tuple=True)
            h = torch.relu(x[tok] @ up.T) ** 2
            y = h @ dn.T
            nxt.index_add_(0, tok, y * wl[tok, slot][:, None])
        x = nxt
    return x


def _expert_dev(bank, l, e):
    cb, sb = bank.up_code_bytes, bank.up_scale_bytes
    db, ds = bank.dn_code_bytes, bank.dn_scale_bytes
    g = bank.globals[l][e].cpu().numpy()
    up = (bank.up_codes[l][e * cb:(e + 1) * cb], bank.up_scales[l][e * sb:(e + 1) * sb], float(g[1]))
    dn = (bank.dn_codes[l][e * db:(e + 1) * db], bank.dn_scales[l][e * ds:(e + 1) * ds], float(g[0]))
    return up, dn


@pytest.mark.parametrize("ksplit", [1, 2])
def test_config4_batch32_all_layers_within_tolerance(bench_bank, cuda, ksplit):
    from ervf_b200.moe import MoEDecoder

    dec = MoEDecoder(bench_bank, TOP_K)
    dec.batch_ksplit = ksplit
    T = 32
    g = torch.Generator(device=cuda)
    g.manual_seed(7)  # bench.py batched_decode inputs
    # bench.py's batch-32 inputs, the hidden states scaled by 1/16 so that the
    # unnormalised recurrence stays finite through the 24 layers
    xb = torch.randn(T, HIDDEN, generator=g, device=cuda) * (1.0 / 16.0)
    rb = torch.randn(N_LAYERS, T, N_EXPERTS, generator=g, device=cuda)
    y = dec.step_batch(xb, rb).clone()
    torch.cuda.synchronize(cuda)
    ids = dec.bids.view(N_LAYERS, T, TOP_K)
    w = dec.bw.view(N_LAYERS, T, TOP_K)
    want = _float64_batch_recurrence(bench_bank, xb, ids, w)
    assert torch.isfinite(want).all()
    err = rel_l2(y.cpu().numpy(), want.cpu().numpy())
    assert err <= 1e-3, err
    # the layers' contributions alone (x_24 - x_0) hold the same tolerance
    moe_err = rel_l2((y - xb).cpu().numpy(), (want - xb.to(torch.float64)).cpu().numpy())
    assert moe_err <= 1e-3, moe_err
