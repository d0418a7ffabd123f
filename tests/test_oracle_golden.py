"""The CPU oracle against golden outputs of the REFERENCE's own CUDA kernels
(tests/golden/gemv_reference.npz, produced on a B200 by
``tests/golden/make_golden.py gemv`` from oracle/_ref/libervf_ref.so), and
properties of the reduction tree that the golden cases cannot show."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import bits_equal, random_nvfp4, rel_l2, x_regime

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
from make_golden import CONFIG0_CASES, GEMV_CASES, case_inputs  # noqa: E402


@pytest.mark.parametrize("i", range(len(GEMV_CASES)))
def test_oracle_matches_reference_kernel_golden(oracle, i):
    rows, cols, seed, regime, relu2, width, full = GEMV_CASES[i]
    g = np.load(HERE / "golden" / "gemv_reference.npz")[f"case{i}"]
    codes, scales, gs, x = case_inputs(i)
    tree = oracle.TREE_LEGACY if width == 256 else oracle.TREE_ERVF
    got = oracle.nvfp4_gemv(codes, scales, x, gs, rows, cols, apply_relu2=bool(relu2), tree=tree)
    assert bits_equal(got, g)


@pytest.mark.parametrize("key,width,relu2", CONFIG0_CASES)
def test_oracle_matches_reference_kernel_on_config0(oracle, key, width, relu2):
    """BASELINE config 0's exact inputs: the oracle equals the reference's
    ERVF-16 (and legacy) kernel output stored from a B200 run."""
    from ervf_b200.formats import config0_inputs

    gold = np.load(HERE / "golden" / "gemv_reference.npz")
    codes, scales, g, x = config0_inputs()
    tree = oracle.TREE_LEGACY if width == 256 else oracle.TREE_ERVF
    got = oracle.nvfp4_gemv(codes, scales, x, g, 1856, 2688, apply_relu2=bool(relu2), tree=tree)
    assert bits_equal(got, gold[key])


def test_oracle_close_to_float64_dequant(oracle):
    from ervf_b200.formats import dequantize

    rows, cols = 64, 2688
    codes, scales, g = random_nvfp4(rows, cols, seed=5)
    x = x_regime(cols, "random", seed=6)
    want = dequantize(codes, scales, g, rows, cols) @ x.astype(np.float64)
    assert rel_l2(oracle.nvfp4_gemv(codes, scales, x, g, rows, cols), want) < 1e-6


def test_chain_order_matters(oracle):
    """Changing the reduction order changes bits: the oracle's chain/tree
    order is observable (fp addition is not associative)."""
    rows, cols = 8, 4096
    codes, scales, g = random_nvfp4(rows, cols, seed=8)
    x = x_regime(cols, "adversarial", seed=9)
    a = oracle.nvfp4_gemv(codes, scales, x, g, rows, cols)
    deq = oracle.dequant_f32(codes, scales, g, rows, cols)
    b = np.array([np.float32(np.sum(deq[r].astype(np.float32) * x, dtype=np.float32))
                  for r in range(rows)])
    assert not bits_equal(a, b)


def test_legacy_and_ervf_trees_differ_only_in_zero_sign(oracle):
    rows, cols = 4, 2048
    codes = np.full(rows * cols // 2, 0x99, np.uint8)
    scales = np.full(rows * cols // 16, 0x01, np.uint8)
    x = np.full(cols, 1e-40, np.float32)
    e = oracle.nvfp4_gemv(codes, scales, x, np.float32(1e-30), rows, cols, tree=oracle.TREE_ERVF)
    l = oracle.nvfp4_gemv(codes, scales, x, np.float32(1e-30), rows, cols, tree=oracle.TREE_LEGACY)
    assert np.all(np.signbit(e)) and not np.any(np.signbit(l)) and np.all(e == l)
    codes, scales, g = random_nvfp4(16, 2688, seed=1)
    x = x_regime(2688, "random", seed=1)
    assert bits_equal(oracle.nvfp4_gemv(codes, scales, x, g, 16, 2688, tree=oracle.TREE_ERVF),
                      oracle.nvfp4_gemv(codes, scales, x, g, 16, 2688, tree=oracle.TREE_LEGACY))


def test_masked_down_equals_row_major_within_tolerance(oracle):
    """Panel-major masked down sums in another order than the row-major GEMV:
    same value to fp32 rounding (s5_masked_smoke.py:81-128 used rel-L2 < 1e-6)."""
    hidden, inter = 256, 128
    codes, scales, g = random_nvfp4(hidden, inter, seed=2)
    act = np.maximum(x_regime(inter, "zero_heavy", seed=3), 0) ** 2
    bank = oracle.panel_major(codes, scales, hidden, inter)
    a = oracle.down_masked(bank, act, g, hidden, inter, 8)
    b = oracle.nvfp4_gemv(codes, scales, act, g, hidden, inter)
    assert rel_l2(a, b) < 1e-6


def test_panel_major_is_a_permutation(oracle):
    hidden, inter = 64, 48
    r = np.random.default_rng(0)
    codes = r.integers(0, 256, hidden * inter // 2, dtype=np.uint8)
    scales = r.integers(0, 256, hidden * inter // 16, dtype=np.uint8)
    bank = oracle.panel_major(codes, scales, hidden, inter)
    assert bank.size == codes.size + scales.size
    nib = np.empty((hidden, inter), np.uint8)
    c = codes.reshape(hidden, inter // 2)
    nib[:, 0::2], nib[:, 1::2] = c & 15, c >> 4
    stride = hidden + 16 * (hidden // 2)
    for p in range(inter // 16):
        blk = bank[p * stride:(p + 1) * stride]
        assert np.array_equal(blk[:hidden], scales.reshape(hidden, inter // 16)[:, p])
        for col in range(16):
            seg = blk[hidden + col * (hidden // 2):hidden + (col + 1) * (hidden // 2)]
            back = np.empty(hidden, np.uint8)
            back[0::2], back[1::2] = seg & 15, seg >> 4
            assert np.array_equal(back, nib[:, 16 * p + col])
