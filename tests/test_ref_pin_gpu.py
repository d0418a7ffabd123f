"""Pins the CPU oracle (and the product) to the REFERENCE's own CUDA kernels,
compiled for sm_100a from kennydd001/ervf's kernel sources by
oracle/build_ref.py and run on the same inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import REGIMES, bits_equal, random_nvfp4, x_regime

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(cuda):
    import ref as r

    if not r.available():
        pytest.skip("oracle/_ref/libervf_ref.so not built (needs the reference tree at build time)")
    return r


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def ref_gemv(ref, fused, width, codes, scales, x, g, rows, cols, relu2=False, out_scale=1.0):
    dev = fused.device
    out = torch.full((rows,), float("nan"), device=dev)
    c, s, xd = _t(codes, dev), _t(scales, dev), _t(x, dev)
    ref.call(ref.ervf_fn(width), c.data_ptr(), s.data_ptr(), fused.e2m1.data_ptr(),
             fused.e4m3.data_ptr(), xd.data_ptr(), out.data_ptr(), float(g), rows, cols,
             int(relu2), float(out_scale), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("rows,cols", [(1856, 2688), (2688, 1856), (1536, 2048), (2048, 768),
                                       (37, 2688)])
def test_oracle_equals_reference_kernels(ref, fused, oracle, rows, cols):
    codes, scales, g = random_nvfp4(rows, cols, seed=rows + 3 * cols, nan_scales=True)
    for regime in REGIMES:
        x = x_regime(cols, regime, seed=len(regime))
        for relu2 in (False, True):
            want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2)
            for width in (4, 8, 16, 32):
                got = ref_gemv(ref, fused, width, codes, scales, x, g, rows, cols, relu2)
                assert bits_equal(got, want), (regime, relu2, width)
            legacy = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2,
                                       tree=oracle.TREE_LEGACY)
            assert bits_equal(ref_gemv(ref, fused, 256, codes, scales, x, g, rows, cols, relu2),
                              legacy)


def test_product_equals_reference_kernel(ref, fused):
    rows, cols = 1856, 2688
    codes, scales, g = random_nvfp4(rows, cols, seed=77)
    x = x_regime(cols, "bf16", seed=1)
    want = ref_gemv(ref, fused, 16, codes, scales, x, g, rows, cols, True)
    out = torch.zeros(rows, device=fused.device)
    fused.gemv_into(out, _t(codes, fused.device), _t(scales, fused.device), _t(x, fused.device), g,
                    rows, cols, apply_relu2=True)
    torch.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), want)


def _product(fused, codes, scales, x, g, rows, cols, relu2, width=0, use_ervf=True):
    dev = fused.device
    fused.ervf_width, fused.use_ervf = width, use_ervf
    out = torch.full((rows,), float("nan"), device=dev)
    fused.gemv_into(out, _t(codes, dev), _t(scales, dev), _t(x, dev), g, rows, cols,
                    apply_relu2=relu2)
    torch.cuda.synchronize()
    fused.ervf_width, fused.use_ervf = 0, True
    return out.cpu().numpy()


def test_config0_exact_inputs_against_reference_kernels(ref, fused, oracle):
    from ervf_b200.formats import config0_inputs

    rows, cols = 1856, 2688
    codes, scales, g, x = config0_inputs()
    for relu2 in (False, True):
        want = ref_gemv(ref, fused, 16, codes, scales, x, g, rows, cols, relu2)
        for width in (4, 8, 32):
            assert bits_equal(ref_gemv(ref, fused, width, codes, scales, x, g, rows, cols, relu2),
                              want), width
        assert bits_equal(oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2), want)
        for width in (0, 4, 8, 16, 32):
            assert bits_equal(_product(fused, codes, scales, x, g, rows, cols, relu2, width), want), width
        legacy = ref_gemv(ref, fused, 256, codes, scales, x, g, rows, cols, relu2)
        assert bits_equal(_product(fused, codes, scales, x, g, rows, cols, relu2, use_ervf=False),
                          legacy)


@pytest.mark.parametrize("rows,cols", [(1856, 2688), (2688, 1856), (2048, 768), (37, 2688),
                                       (64, 4096)])
def test_full_scale_byte_range_against_reference_kernels(ref, fused, oracle, rows, cols):
    """Every scale byte class -- negative, subnormal, large, zero, NaN -- through
    the reference kernels, the oracle and the product."""
    codes, scales, g = random_nvfp4(rows, cols, seed=rows + 5 * cols, full_range=True)
    for regime in ("random", "adversarial"):
        x = x_regime(cols, regime, seed=rows)
        for relu2 in (False, True):
            want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2)
            for width in (4, 8, 16, 32):
                assert bits_equal(ref_gemv(ref, fused, width, codes, scales, x, g, rows, cols, relu2),
                                  want), (regime, relu2, width)
            legacy = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2,
                                       tree=oracle.TREE_LEGACY)
            assert bits_equal(ref_gemv(ref, fused, 256, codes, scales, x, g, rows, cols, relu2), legacy)
            for width in (0, 16):
                assert bits_equal(_product(fused, codes, scales, x, g, rows, cols, relu2, width),
                                  want), (regime, relu2, width)


@pytest.mark.parametrize("rows,cols", [(3712, 2688), (2688, 3712), (131072, 2688)])
def test_shared_expert_and_lm_head_shapes_against_reference(ref, fused, oracle, rows, cols):
    """The runtime's other NVFP4 GEMVs (runtime.py:510-515 shared expert up /
    down, :827-829 lm_head) through the same kernel: product == reference
    ERVF-16 kernel bit for bit (cols 3712 runs the B200 schedule with 52
    second-round chain groups); the oracle on the first rows."""
    codes, scales, g = random_nvfp4(rows, cols, seed=rows + cols, full_range=True)
    x = x_regime(cols, "bf16", seed=3)
    for relu2 in ((False, True) if rows < 100000 else (False,)):
        want = ref_gemv(ref, fused, 16, codes, scales, x, g, rows, cols, relu2)
        assert bits_equal(_product(fused, codes, scales, x, g, rows, cols, relu2), want)
        n = min(rows, 4096)
        o = oracle.nvfp4_gemv(codes[:n * cols // 2], scales[:n * cols // 16], x, g, n, cols,
                              apply_relu2=relu2)
        assert bits_equal(o, want[:n])


def test_bf16_oracle_equals_reference(ref, oracle, cuda):
    rows, cols = 512, 2688
    r = np.random.default_rng(4)
    W = (r.standard_normal((rows, cols)).astype(np.float32) * 0.02).view(np.uint32) >> 16
    W = W.astype(np.uint16)
    x = r.standard_normal(cols).astype(np.float32)
    out = torch.zeros(rows, device=cuda)
    Wd, xd = _t(W, cuda), _t(x, cuda)
    ref.call("ref_gemv_bf16", Wd.data_ptr(), xd.data_ptr(), out.data_ptr(),
             rows, cols, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), oracle.bf16_gemv(W, x, rows, cols)[0])


def test_f32_oracle_equals_reference(ref, oracle, cuda):
    """The router projection: the oracle's gemv_f32 restatement against the
    reference's own gemv_f32 kernel (gpu_kernels.py:51-74), and the library's
    fused router against both."""
    from ervf_b200 import FusedNVFP4, GPUKernels

    for rows, cols, seed in ((128, 2688, 5), (37, 1000, 6)):
        r = np.random.default_rng(seed)
        W = r.standard_normal((rows, cols)).astype(np.float32) * 0.02
        x = r.standard_normal(cols).astype(np.float32)
        out = torch.zeros(rows, device=cuda)
        Wd, xd = _t(W, cuda), _t(x, cuda)
        ref.call("ref_gemv_f32", Wd.data_ptr(), xd.data_ptr(), out.data_ptr(),
                 rows, cols, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        want = oracle.f32_gemv(W, x, rows, cols)
        assert bits_equal(out.cpu().numpy(), want)
        if cols % 4 == 0:
            mine = torch.zeros(rows, device=cuda)
            GPUKernels(device=cuda).mv_f32(mine, Wd, xd, rows, cols)
            torch.cuda.synchronize()
            assert bits_equal(mine.cpu().numpy(), want)


def test_masked_down_oracle_equals_reference(ref, fused, oracle, cuda):
    hidden, inter = 2688, 1856
    codes, scales, g = random_nvfp4(hidden, inter, seed=12)
    bank = oracle.panel_major(codes, scales, hidden, inter)
    act = x_regime(inter, "zero_heavy", seed=3)
    st = fused.alloc_masked_state(hidden, inter)
    out = torch.zeros(hidden, device=cuda)
    bank_d = _t(bank, cuda)
    act_d = _t(act, cuda)
    ref.call("ref_down_masked", out.data_ptr(), bank_d.data_ptr(), act_d.data_ptr(),
             st["masks"].data_ptr(), st["plist"].data_ptr(), st["pcount"].data_ptr(),
             st["nz"].data_ptr(), st["nzc"].data_ptr(), st["partials"].data_ptr(),
             fused.e2m1.data_ptr(), fused.e4m3.data_ptr(), float(g), hidden, inter, 8,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = oracle.down_masked(bank, act, g, hidden, inter, 8)
    assert bits_equal(out.cpu().numpy(), want)


def test_router_and_lru_oracle_equal_reference(ref, oracle, cuda):
    r = np.random.default_rng(9)
    n, k = 128, 6
    state_ref = None
    for tok in range(20):
        rlog = r.standard_normal(n).astype(np.float32)
        bias = np.zeros(n, np.float32)
        ids = torch.zeros(k, dtype=torch.int32, device=cuda)
        w = torch.zeros(k, device=cuda)
        rlog_d, bias_d = _t(rlog, cuda), _t(bias, cuda)  # keep alive across the launch
        ref.call("ref_route_topk", rlog_d.data_ptr(), bias_d.data_ptr(),
                 ids.data_ptr(), w.data_ptr(), n, k, 1.0, 0, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        oid, ow = oracle.route_topk(rlog, bias, k)
        assert np.array_equal(ids.cpu().numpy(), oid)
        np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=3e-7, atol=0)
        if state_ref is None:
            cap = 16
            state_ref = {kk: torch.full((sz,), -1, dtype=torch.int32, device=cuda)
                         for kk, sz in (("slot_of", n), ("expert_of", cap), ("last_used", cap))}
            state_ref["state2"] = torch.zeros(2, dtype=torch.int32, device=cuda)
            state_ref["stats2"] = torch.zeros(2, dtype=torch.int32, device=cuda)
            state_o = {kk: v.cpu().numpy().copy() for kk, v in state_ref.items()}
        slots = torch.zeros(k, dtype=torch.int32, device=cuda)
        need = torch.zeros(k, dtype=torch.int32, device=cuda)
        ref.call("ref_cache_assign", state_ref["slot_of"].data_ptr(), state_ref["expert_of"].data_ptr(),
                 state_ref["last_used"].data_ptr(), state_ref["state2"].data_ptr(), ids.data_ptr(),
                 slots.data_ptr(), need.data_ptr(), state_ref["stats2"].data_ptr(), 16, k,
                 torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        os_, on = oracle.cache_assign(state_o, oid, 16, k)
        assert np.array_equal(slots.cpu().numpy(), os_) and np.array_equal(need.cpu().numpy(), on)
        for kk in state_o:
            assert np.array_equal(state_ref[kk].cpu().numpy(), state_o[kk]), kk
