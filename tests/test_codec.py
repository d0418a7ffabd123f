"""Codec known-answer tests, re-hosted from the reference
(tests/lightningstream_nemotron/test_nvfp4.py:19-133) onto this package's
tables (``ervf_b200.formats``) and the oracle's C tables, plus the golden
tables generated from the reference's own nvfp4.py
(tests/golden/make_golden.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from ervf_b200 import formats

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_e2m1_magnitudes_match_published_set():
    assert np.unique(np.abs(formats.e2m1_table())).tolist() == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def test_e2m1_sign_symmetry():
    t = formats.e2m1_table()
    assert np.array_equal(t[:8], -t[8:])


def test_e4m3_nan_only_at_7f_ff_and_device_maps_to_zero():
    raw = formats.e4m3_table()
    assert np.flatnonzero(np.isnan(raw)).tolist() == [0x7F, 0xFF]
    dev = formats.e4m3_device_table()
    assert dev[0x7F] == 0.0 and dev[0xFF] == 0.0 and not np.signbit(dev[0xFF])


def test_e4m3_known_values():
    raw = formats.e4m3_table()
    assert np.nanmax(raw) == 448.0
    assert raw[0x01] == 2.0 ** -9
    assert raw[0x38] == 1.0 and raw[0x3C] == 1.5
    assert raw[0x80] == 0.0 and np.signbit(raw[0x80])


def test_oracle_tables_equal_package_tables(oracle):
    e2m1, dev, raw = oracle.luts()
    assert np.array_equal(e2m1.view(np.uint32), formats.e2m1_table().view(np.uint32))
    assert np.array_equal(dev.view(np.uint32), formats.e4m3_device_table().view(np.uint32))
    nan = np.isnan(raw)
    assert np.array_equal(nan, np.isnan(formats.e4m3_table()))
    assert np.array_equal(raw[~nan], formats.e4m3_table()[~nan])


def test_tables_equal_reference_golden():
    g = np.load(GOLDEN / "codec_tables.npz")
    assert np.array_equal(g["e2m1"], formats.e2m1_table().astype(np.float64))
    raw = g["e4m3"]
    nan = np.isnan(raw)
    assert np.array_equal(nan, np.isnan(formats.e4m3_table()))
    assert np.array_equal(raw[~nan], formats.e4m3_table()[~nan].astype(np.float64))


def test_nibble_order_low_first():
    w = np.zeros((1, 16), np.float32)
    w[0, 0], w[0, 1] = 0.5, 1.0
    packed, scales, g = formats.quantize_nvfp4(w)
    # the block amax 1.0 maps to 6: element 0 -> 3.0 (code 5) in the LOW
    # nibble, element 1 -> 6.0 (code 7) in the high nibble
    assert packed[0, 0] == (5 | (7 << 4))
    assert formats.e4m3_table()[scales[0, 0]] * g == np.float32(1.0 / 6.0)


def test_dequantize_matches_reference_golden():
    g = np.load(GOLDEN / "codec_tables.npz")
    out = formats.dequantize(g["dq_codes"], g["dq_scales"], float(g["dq_g"]), 1,
                             g["dq_codes"].size * 2)
    assert np.array_equal(out.reshape(-1), g["dq_out"])


def test_quantiser_round_trip_is_representable_and_close():
    w = formats.synthetic_weight(64, 256, seed=0)
    codes, scales, g = formats.quantize_nvfp4(w)
    dq = formats.dequantize(codes, scales, g, 64, 256)
    assert np.linalg.norm(dq - w) / np.linalg.norm(w) < 0.15
    # every dequantised value is code * scale * g of its block
    allowed_mag = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0}
    s = formats.e4m3_table()[scales].astype(np.float64) * float(g)
    ratio = np.abs(dq.reshape(64, 16, 16)) / s[:, :, None]
    assert set(np.unique(np.round(ratio, 12)).tolist()) <= allowed_mag


def test_quantiser_torch_equals_numpy():
    torch = pytest.importorskip("torch")
    w = formats.synthetic_weight(48, 512, seed=3)
    c1, s1, g1 = formats.quantize_nvfp4(w)
    c2, s2, g2 = formats.quantize_nvfp4_torch(torch.from_numpy(w))
    assert np.array_equal(c1, c2.numpy()) and np.array_equal(s1, s2.numpy())
    assert np.float32(g1) == np.float32(g2.item())
