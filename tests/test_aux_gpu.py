"""BF16 GEMV, device router, device LRU, expert fetch and the masked down
path on the GPU against the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bits_equal, random_nvfp4, rel_l2, x_regime

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _bf16_bits(a):
    return (np.ascontiguousarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("rows,cols,batch", [(4096, 2688, 1), (2688, 4096, 1), (4096, 2688, 8),
                                             (300, 2696, 3), (33, 8, 1)])
def test_bf16_gemv_bit_exact_and_tolerance(cuda, oracle, rows, cols, batch):
    from ervf_b200 import GPUKernels

    r = np.random.default_rng(rows + cols + batch)
    W = _bf16_bits(r.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    x = r.standard_normal(batch * cols).astype(np.float32)
    out = torch.zeros(batch * rows, device=cuda)
    GPUKernels().mv_bf16_batched(out, _t(W, cuda), _t(x, cuda), rows, cols, batch)
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(batch, rows)
    assert bits_equal(got, oracle.bf16_gemv(W, x, rows, cols, batch))
    Wf = torch.from_numpy((W.astype(np.uint32) << 16).view(np.float32))
    ref = (torch.from_numpy(x.reshape(batch, cols)) @ Wf.T).numpy()
    assert rel_l2(got, ref) <= 1e-3


def test_route_topk_matches_oracle(fused, oracle, cuda):
    r = np.random.default_rng(2)
    for n, k, bias_on, bad in ((128, 6, False, 0), (128, 8, True, 0), (128, 6, False, 1),
                               (64, 4, True, 0)):
        rlog = r.standard_normal(n).astype(np.float32)
        bias = (r.standard_normal(n) * 0.1).astype(np.float32) if bias_on else np.zeros(n, np.float32)
        ids = torch.zeros(k, dtype=torch.int32, device=cuda)
        w = torch.zeros(k, device=cuda)
        fused.route_topk(_t(rlog, cuda), _t(bias, cuda), ids, w, n, k, 2.5, bad_pick=bad)
        torch.cuda.synchronize()
        oid, ow = oracle.route_topk(rlog, bias, k, 2.5, bad)
        assert np.array_equal(ids.cpu().numpy(), oid)
        np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=3e-7)


@pytest.mark.parametrize("n,hidden,k,bias,bad", [(128, 2688, 6, False, 0), (128, 2688, 6, True, 1),
                                                 (200, 1024, 8, True, 0), (33, 64, 3, False, 0)])
def test_route_gemv_topk_matches_oracle(fused, oracle, cuda, n, hidden, k, bias, bad):
    """Router projection (gemv_f32) + sigmoid top-k in one launch equals the
    reference pair mv_f32 + route_topk (runtime.py:710-713): rlog, ids and
    weights bit for bit, over repeated calls (the counter stays zero)."""
    from ervf_b200 import _lib

    r = np.random.default_rng(n + hidden + k)
    gw = r.standard_normal((n, hidden)).astype(np.float32) * 0.05
    gb = (r.standard_normal(n).astype(np.float32) * 0.1) if bias else None
    gwd = _t(gw, cuda)
    gbd = _t(gb, cuda) if bias else None
    for call in range(3):
        x = r.standard_normal(hidden).astype(np.float32)
        rlog = torch.zeros(n, device=cuda)
        ids = torch.zeros(k, dtype=torch.int32, device=cuda)
        w = torch.zeros(k, device=cuda)
        fused.route_gemv_topk(rlog, gwd, _t(x, cuda), gbd, ids, w, n, hidden, k, 1.5, bad_pick=bad,
                              flags=_lib.LAUNCH_PDL if call == 2 else 0)
        torch.cuda.synchronize()
        want_log = oracle.f32_gemv(gw, x, n, hidden)
        oid, ow = oracle.route_topk(want_log, gb if bias else np.zeros(n, np.float32), k, 1.5, bad)
        assert bits_equal(rlog.cpu().numpy(), want_log)
        assert np.array_equal(ids.cpu().numpy(), oid)
        # the weights use CUDA expf (the oracle's libm expf may differ by an
        # ulp): within tolerance of the oracle, bit-equal to the standalone
        # device router on the same logits
        np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=3e-7)
        ids1 = torch.zeros(k, dtype=torch.int32, device=cuda)
        w1 = torch.zeros(k, device=cuda)
        fused.route_topk(rlog, gbd if bias else torch.zeros(n, device=cuda), ids1, w1, n, k, 1.5,
                         bad_pick=bad)
        torch.cuda.synchronize()
        assert torch.equal(ids1, ids) and torch.equal(w1.view(torch.int32), w.view(torch.int32))
    assert int(fused._rcounter.item()) == 0


def test_route_topk_batched_matches_per_layer(fused, oracle, cuda):
    r = np.random.default_rng(12)
    for n, k in ((128, 6), (128, 8), (200, 6), (512, 4)):
        L = 24
        rl = r.standard_normal((L, n)).astype(np.float32)
        bias = (r.standard_normal((L, n)) * 0.05).astype(np.float32)
        ids = torch.zeros(L, k, dtype=torch.int32, device=cuda)
        w = torch.zeros(L, k, device=cuda)
        rd, bd = _t(rl, cuda), _t(bias, cuda)
        fused.route_topk_batched(rd, bd, ids, w, L, n, k, 1.0, 0, n)
        torch.cuda.synchronize()
        for l in range(L):
            oid, ow = oracle.route_topk(rl[l], bias[l], k)
            assert np.array_equal(ids[l].cpu().numpy(), oid), (n, k, l)
            np.testing.assert_allclose(w[l].cpu().numpy(), ow, rtol=3e-7)
            one_ids = torch.zeros(k, dtype=torch.int32, device=cuda)
            one_w = torch.zeros(k, device=cuda)
            fused.route_topk(rd[l], bd[l], one_ids, one_w, n, k, 1.0)
            torch.cuda.synchronize()
            assert torch.equal(one_ids, ids[l]) and torch.equal(one_w, w[l])


def test_route_topk_ties_pick_lowest_index(fused, cuda):
    rlog = np.zeros(128, np.float32)
    rlog[[5, 9, 77]] = 3.0
    ids = torch.zeros(4, dtype=torch.int32, device=cuda)
    w = torch.zeros(4, device=cuda)
    fused.route_topk(_t(rlog, cuda), torch.zeros(128, device=cuda), ids, w, 128, 4, 1.0)
    torch.cuda.synchronize()
    assert ids.cpu().tolist() == [5, 9, 77, 0]


def test_cache_assign_and_fetch_track_oracle(fused, oracle, cuda):
    n_experts, cap, k = 32, 10, 6
    code_bytes, scale_bytes = 4096, 512
    r = np.random.default_rng(8)
    bank_c = r.integers(0, 256, n_experts * code_bytes, dtype=np.uint8)
    bank_s = r.integers(0, 256, n_experts * scale_bytes, dtype=np.uint8)
    bc, bs = _t(bank_c, cuda), _t(bank_s, cuda)
    cache_c = torch.zeros(cap * code_bytes, dtype=torch.uint8, device=cuda)
    cache_s = torch.zeros(cap * scale_bytes, dtype=torch.uint8, device=cuda)
    dev = fused.alloc_device_cache(n_experts, cap, k, np.zeros((n_experts, 2), np.float32))
    st = {kk: dev[kk].cpu().numpy().copy() for kk in ("slot_of", "expert_of", "last_used", "state2",
                                                       "stats2")}
    for tok in range(40):
        ids_h = r.choice(12, size=k, replace=False).astype(np.int32)
        dev["ids"].copy_(_t(ids_h, cuda))
        fused.cache_assign(dev, dev["ids"], cap, k)
        fused.cache_fetch(bc.data_ptr(), bs.data_ptr(), cache_c, cache_s, dev, code_bytes,
                          scale_bytes, k)
        torch.cuda.synchronize()
        slots, need = oracle.cache_assign(st, ids_h, cap, k)
        assert np.array_equal(dev["slots"].cpu().numpy(), slots)
        assert np.array_equal(dev["need"].cpu().numpy(), need)
        cc = cache_c.cpu().numpy()
        for s, e in enumerate(ids_h):
            sl = slots[s]
            assert np.array_equal(cc[sl * code_bytes:(sl + 1) * code_bytes],
                                  bank_c[e * code_bytes:(e + 1) * code_bytes])
    assert np.array_equal(dev["stats2"].cpu().numpy(), st["stats2"])


@pytest.mark.parametrize("nchunks", [8, 3])
def test_masked_down_matches_oracle(fused, oracle, cuda, nchunks):
    hidden, inter = 2688, 1856
    codes, scales, g = random_nvfp4(hidden, inter, seed=31)
    bank = oracle.panel_major(codes, scales, hidden, inter)
    # the device repack equals the oracle's restatement of down_panel_major
    blk = torch.zeros(bank.size, dtype=torch.uint8, device=cuda)
    from ervf_b200 import _lib
    cd, sd = _t(codes, cuda), _t(scales, cuda)  # alive until the launch has run
    _lib.call("ervf_panel_major", cd.data_ptr(), sd.data_ptr(), blk.data_ptr(), hidden, inter,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(blk.cpu().numpy(), bank)
    st = fused.alloc_masked_state(hidden, inter)
    for regime in ("zero_heavy", "random"):
        act = x_regime(inter, regime, seed=nchunks)
        act = np.maximum(act, 0) ** 2
        out = torch.zeros(hidden, device=cuda)
        fused.down_masked_into(out, blk.data_ptr(), _t(act, cuda), st, g, hidden, inter,
                               nchunks=nchunks)
        torch.cuda.synchronize()
        assert bits_equal(out.cpu().numpy(), oracle.down_masked(bank, act, g, hidden, inter, nchunks))
