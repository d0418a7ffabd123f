"""Shared fixtures.  Tests marked ``gpu`` need a CUDA device (a B200) and the
built libraries; everything else runs on CPU."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.build()
    return o


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ervf_b200 import build

    build.build()
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def fused(cuda):
    from ervf_b200 import FusedNVFP4

    return FusedNVFP4()


def rng(seed):
    return np.random.default_rng(seed)


def random_nvfp4(rows, cols, seed, nan_scales=False, full_range=False):
    """Random codes and block scales (bytes), as the reference's verifiers use
    (e1f21_independent_verify.py:173-176).  By default the scale bytes avoid
    huge values (0x20-0x4F); full_range=True draws every byte 0x00-0xFF:
    negative scales (0x80-0xFE), subnormal (0x01-0x07), large (0x50-0x7E),
    zero and the NaN bytes 0x7F / 0xFF."""
    r = rng(seed)
    codes = r.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    if full_range:
        scales = r.integers(0, 256, size=rows * cols // 16, dtype=np.uint8)
        # make sure every class is present even in small cases
        special = np.array([0x00, 0x01, 0x07, 0x50, 0x7E, 0x7F, 0x80, 0x81, 0xFE, 0xFF], np.uint8)
        scales[:min(special.size, scales.size)] = special[:scales.size]
        g = np.float32(r.uniform(1e-4, 1e-2))
        return codes, scales, g
    scales = r.integers(0x20, 0x50, size=rows * cols // 16, dtype=np.uint8)
    if nan_scales:
        idx = r.choice(scales.size, size=max(1, scales.size // 50), replace=False)
        scales[idx] = r.choice(np.array([0x7F, 0xFF], np.uint8), size=idx.size)
    g = np.float32(r.uniform(1e-4, 1e-2))
    return codes, scales, g


def x_regime(cols, regime, seed):
    """Activation regimes of the reference's exactness sweep
    (nervf01_geometry_audit.py:458-467)."""
    r = rng(seed)
    if regime == "random":
        return r.standard_normal(cols).astype(np.float32)
    if regime == "adversarial":
        return (r.standard_normal(cols) * 10.0 ** r.integers(-8, 8, cols)).astype(np.float32)
    if regime == "zero_heavy":
        return np.where(r.random(cols) < 0.9, 0.0, r.standard_normal(cols)).astype(np.float32)
    if regime == "dense":
        return (r.random(cols) + 0.5).astype(np.float32)
    if regime == "bf16":
        x = r.standard_normal(cols).astype(np.float32)
        return (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    raise ValueError(regime)


REGIMES = ["random", "adversarial", "zero_heavy", "dense"]


def bits_equal(a, b) -> bool:
    a = np.ascontiguousarray(a, np.float32).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and bool(np.array_equal(a, b))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    n = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (n if n > 0 else 1.0))


def dequant_torch(codes, scales, g, rows, cols, dtype=None):
    """float64 (default) dequantisation on the tensors' device: E2M1 code x
    E4M3 block scale (NaN bytes -> 0, as the kernels' tables) x global scale.
    A tolerance reference for the tensor-core paths."""
    import torch

    from ervf_b200.formats import e2m1_table, e4m3_device_table

    dtype = dtype or torch.float64
    dev = codes.device
    e2 = torch.from_numpy(e2m1_table()).to(dev, dtype)
    e4 = torch.from_numpy(e4m3_device_table()).to(dev, dtype)
    c = codes.reshape(rows, cols // 2).long()
    nib = torch.stack([c & 15, c >> 4], dim=2).reshape(rows, cols)
    s = e4[scales.reshape(rows, cols // 16).long()].repeat_interleave(16, dim=1)
    return e2[nib] * s * float(g)
