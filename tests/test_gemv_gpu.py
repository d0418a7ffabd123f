"""NVFP4 GEMV parity on the GPU: the product (through the C ABI, via the
reference-shaped ``FusedNVFP4`` shim and directly) against the CPU oracle,
bit for bit, across shapes, widths, epilogues and activation regimes."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import REGIMES, bits_equal, random_nvfp4, x_regime

pytestmark = pytest.mark.gpu

SHAPES = [
    (1856, 2688),   # config 0: routed up_proj
    (2688, 1856),   # routed down_proj
    (1536, 2048),   # Qwen fused gate+up
    (2048, 768),    # Qwen down
    (37, 2688),     # ragged row tile
    (1, 32),
    (17, 16),       # smallest cols, width-32 fallback
    (33, 2704),     # cols % 32 == 16 -> width-32 fallback
    (64, 4096),
    (24, 8192),     # cols > 4096 -> width-32 fallback
    (96, 3712),     # shared-expert down: 52 second-round chain groups
]


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def run_product(fused, codes, scales, x, g, rows, cols, relu2=False, out_scale=1.0, width=0,
                use_ervf=True, device="cuda"):
    fused.ervf_width = width
    fused.use_ervf = use_ervf
    out = torch.full((rows,), float("nan"), device=device)
    fused.gemv_into(out, _dev(codes, device), _dev(scales, device), _dev(x, device), g, rows, cols,
                    apply_relu2=relu2, out_scale=out_scale)
    torch.cuda.synchronize()
    fused.ervf_width, fused.use_ervf = 0, True
    return out.cpu().numpy()


@pytest.mark.parametrize("full_range", [False, True])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_matches_oracle_all_widths(fused, oracle, cuda, rows, cols, full_range):
    codes, scales, g = random_nvfp4(rows, cols, seed=rows * 7 + cols, full_range=full_range)
    x = x_regime(cols, "random", seed=cols)
    want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols)
    for width in (0, 4, 8, 16, 32):
        got = run_product(fused, codes, scales, x, g, rows, cols, width=width, device=cuda)
        assert bits_equal(got, want), f"width {width}: {np.abs(got - want).max()}"


@pytest.mark.parametrize("regime", REGIMES)
@pytest.mark.parametrize("relu2", [False, True])
def test_gemv_regimes_and_epilogue(fused, oracle, cuda, regime, relu2):
    rows, cols = 1856, 2688
    codes, scales, g = random_nvfp4(rows, cols, seed=11)
    x = x_regime(cols, regime, seed=5)
    want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, apply_relu2=relu2)
    got = run_product(fused, codes, scales, x, g, rows, cols, relu2=relu2, device=cuda)
    assert bits_equal(got, want)


def test_gemv_out_scale_and_nan_scales(fused, oracle, cuda):
    rows, cols = 300, 1856
    codes, scales, g = random_nvfp4(rows, cols, seed=3, nan_scales=True)
    x = x_regime(cols, "random", seed=9)
    want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, out_scale=0.37)
    got = run_product(fused, codes, scales, x, g, rows, cols, out_scale=0.37, device=cuda)
    assert bits_equal(got, want)


def test_legacy_tree_differs_only_in_zero_sign(fused, oracle, cuda):
    # tiny products underflow to -0.0 chains; the legacy combine turns an
    # all -0.0 row into +0.0, ERVF keeps -0.0 (fused_nvfp4.py:107-112 vs :397-403)
    rows, cols = 16, 2048  # every one of the 256 chains has work
    codes = np.full(rows * cols // 2, 0x99, np.uint8)  # -0.5 codes
    scales = np.full(rows * cols // 16, 0x01, np.uint8)  # 2^-9
    x = np.full(cols, 1e-40, np.float32)
    g = np.float32(1e-30)
    ervf = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, tree=oracle.TREE_ERVF)
    legacy = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols, tree=oracle.TREE_LEGACY)
    assert np.all(np.signbit(ervf)) and not np.any(np.signbit(legacy))
    assert bits_equal(run_product(fused, codes, scales, x, g, rows, cols, device=cuda), ervf)
    assert bits_equal(run_product(fused, codes, scales, x, g, rows, cols, use_ervf=False,
                                  device=cuda), legacy)


def test_gemv_misaligned_codes_fall_back(fused, oracle, cuda):
    rows, cols = 40, 2688
    codes, scales, g = random_nvfp4(rows, cols, seed=21)
    x = x_regime(cols, "random", seed=2)
    want = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols)
    # 4-byte offset: TMA schedule needs 16-B alignment, the fallback runs
    buf = torch.zeros(codes.size + 4, dtype=torch.uint8, device=cuda)
    buf[4:] = torch.from_numpy(codes).to(cuda)
    sbuf = torch.zeros(scales.size + 1, dtype=torch.uint8, device=cuda)
    sbuf[1:] = torch.from_numpy(scales).to(cuda)
    out = torch.zeros(rows, device=cuda)
    fused.gemv_into(out, buf[4:], sbuf[1:], torch.from_numpy(x).to(cuda), g, rows, cols)
    torch.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), want)


def test_gemv_rejects_bad_shapes(fused, cuda):
    out = torch.zeros(8, device=cuda)
    c = torch.zeros(64, dtype=torch.uint8, device=cuda)
    s = torch.zeros(8, dtype=torch.uint8, device=cuda)
    x = torch.zeros(24, device=cuda)
    with pytest.raises(ValueError):
        fused.gemv_into(out, c, s, x, 1.0, 8, 24)     # cols % 16 != 0
    fused.ervf_width = 12
    with pytest.raises(ValueError):
        fused.gemv_into(out, c, s, x, 1.0, 8, 16)
    fused.ervf_width = 0


def test_gemv_indirect_matches_direct(fused, oracle, cuda):
    rows, cols, n_slots = 1856, 2688, 5
    cb, sb = rows * cols // 2, rows * cols // 16
    recs = [random_nvfp4(rows, cols, seed=100 + i) for i in range(n_slots)]
    cache_c = torch.from_numpy(np.concatenate([r[0] for r in recs])).to(cuda)
    cache_s = torch.from_numpy(np.concatenate([r[1] for r in recs])).to(cuda)
    n_experts = 9
    globals_h = np.random.default_rng(1).uniform(1e-4, 1e-2, (n_experts, 2)).astype(np.float32)
    dev = fused.alloc_device_cache(n_experts, n_slots, 3, globals_h)
    dev["slots"][:] = torch.tensor([4, 0, 2], dtype=torch.int32)
    dev["ids"][:] = torch.tensor([7, 1, 3], dtype=torch.int32)
    x = x_regime(cols, "random", seed=8)
    xd = torch.from_numpy(x).to(cuda)
    for s in range(3):
        slot = int(dev["slots"][s])
        e = int(dev["ids"][s])
        out = torch.zeros(rows, device=cuda)
        fused.gemv_ervf_indirect(out, cache_c, cache_s, dev, s, dev["globals"], 1, xd, rows, cols,
                                 True, cb, sb)
        torch.cuda.synchronize()
        want = oracle.nvfp4_gemv(recs[slot][0], recs[slot][1], x, globals_h[e, 1], rows, cols,
                                 apply_relu2=True)
        assert bits_equal(out.cpu().numpy(), want)


def test_grouped_gemv_c_abi(cuda, oracle):
    from ervf_b200 import _lib

    rows, cols, k = 512, 2688, 6
    recs = [random_nvfp4(rows, cols, seed=300 + i) for i in range(k)]
    xs = [x_regime(cols, "random", seed=400 + i) for i in range(k)]
    dc = [torch.from_numpy(r[0]).to(cuda) for r in recs]
    ds = [torch.from_numpy(r[1]).to(cuda) for r in recs]
    dx = [torch.from_numpy(x).to(cuda) for x in xs]
    do = [torch.zeros(rows, device=cuda) for _ in range(k)]
    P = ctypes.c_void_p * k
    gs = (ctypes.c_float * k)(*[float(r[2]) for r in recs])
    _lib.call("ervf_nvfp4_gemv_grouped", k, P(*[t.data_ptr() for t in dc]),
              P(*[t.data_ptr() for t in ds]), gs, P(*[t.data_ptr() for t in dx]),
              P(*[t.data_ptr() for t in do]), rows, cols, 1, 1.0, 0,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for i in range(k):
        want = oracle.nvfp4_gemv(recs[i][0], recs[i][1], xs[i], recs[i][2], rows, cols,
                                 apply_relu2=True)
        assert bits_equal(do[i].cpu().numpy(), want)
