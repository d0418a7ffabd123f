"""NVFP4 storage formats: E2M1 codes, E4M3 block scales, FP32 global scale.

Format definition (kennydd001/ervf src/moe_lab/lightningstream_nemotron/
nvfp4.py:1-76): E2M1 = 1 sign, 2 exponent (bias 1), 1 mantissa bit, magnitudes
{0, 0.5, 1, 1.5, 2, 3, 4, 6}; E4M3 = 1 sign, 4 exponent (bias 7), 3 mantissa
bits, subnormals 2^-6 * m/8, NaN only at 0x7F / 0xFF, max 448; group size 16;
two codes per byte, low nibble first.  The device tables map the E4M3 NaN
bytes to 0.0 (fused_nvfp4.py:760-762).

The quantiser makes synthetic checkpoints (the real one is not available):
g = max_block_amax / (6 * 448) in fp32, block scale = E4M3-RNE(amax/6 / g),
code = E2M1-RNE(w / (e4m3(scale) * g)), saturating.  The reference has no
rounding encoder (its ``encode_e2m1`` is strict, nvfp4.py:158-185), so this
rule is this project's own; kernel parity never depends on it because both
sides read the same bytes.
"""

from __future__ import annotations

import numpy as np

GROUP = 16
E2M1_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E4M3_MAX = 448.0


def _e4m3_value(b: int) -> float:
    sign = -1.0 if b & 0x80 else 1.0
    e, m = (b >> 3) & 0xF, b & 7
    if e == 0xF and m == 7:
        return float("nan")
    if e == 0:
        return sign * (m / 8.0) * 2.0 ** -6
    return sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)


def e2m1_table() -> np.ndarray:
    return np.array([(-1.0 if c & 8 else 1.0) * E2M1_MAGNITUDES[c & 7] for c in range(16)],
                    dtype=np.float32)


def e4m3_table() -> np.ndarray:
    """Raw decode, NaN at 0x7F / 0xFF."""
    return np.array([_e4m3_value(b) for b in range(256)], dtype=np.float32)


def e4m3_device_table() -> np.ndarray:
    """The decode the kernels use: NaN bytes -> +0.0."""
    return np.nan_to_num(e4m3_table(), nan=0.0).astype(np.float32)


# positive finite E4M3 values, ascending, indexed by byte 0x00..0x7E
_E4M3_POS = e4m3_table()[:0x7F].astype(np.float64)
_E2M1_POS = np.array(E2M1_MAGNITUDES, dtype=np.float64)


def _rne_index(mag: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Index of the nearest table entry to |mag| (float64), ties to the even
    index (= even mantissa LSB), saturating at the top entry."""
    hi = np.searchsorted(table, mag, side="left")
    hi = np.clip(hi, 0, table.size - 1)
    lo = np.clip(hi - 1, 0, table.size - 1)
    d_lo = mag - table[lo]
    d_hi = table[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    idx = np.where(pick_hi, hi, lo)
    return np.where(mag >= table[-1], table.size - 1, idx)


def quantize_nvfp4(w: np.ndarray):
    """fp32 [rows, cols] -> (codes u8 [rows, cols/2], scales u8 [rows, cols/16],
    global_scale float32)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if cols % GROUP:
        raise ValueError("cols must be a multiple of 16")
    blocks = w.reshape(rows, cols // GROUP, GROUP)
    amax = np.abs(blocks).max(axis=2)
    g = np.float32(amax.max()) / np.float32(6.0 * E4M3_MAX)
    if g == 0:
        g = np.float32(1.0)
    target = (amax / np.float32(6.0)).astype(np.float32) / g
    sbytes = _rne_index(target.astype(np.float64), _E4M3_POS).astype(np.uint8)
    denom = (_E4M3_POS[sbytes].astype(np.float32) * g).astype(np.float32)
    safe = np.where(denom == 0, np.float32(1.0), denom)
    q = (blocks / safe[:, :, None]).astype(np.float32)
    mag = _rne_index(np.abs(q).astype(np.float64), _E2M1_POS).astype(np.uint8)
    code = np.where(denom[:, :, None] == 0, 0, mag)
    code = np.where((q < 0) & (code != 0), code | 8, code).astype(np.uint8).reshape(rows, cols)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, sbytes, np.float32(g)


def synthetic_weight(rows: int, cols: int, seed: int) -> np.ndarray:
    """fp32 weights ~ N(0, 0.02) from numpy's default_rng(seed)."""
    return (np.random.default_rng(seed).standard_normal((rows, cols), dtype=np.float32)
            * np.float32(0.02)).astype(np.float32)


def synthetic_nvfp4(rows: int, cols: int, seed: int):
    """Seeded synthetic NVFP4 matrix (codes, scales, g)."""
    return quantize_nvfp4(synthetic_weight(rows, cols, seed))


def config0_inputs():
    """BASELINE config 0 exactly: W [1856 x 2688] ~ N(0, 0.02) from numpy's
    default_rng(0), quantised per 16-element row block (E4M3 block scale =
    block amax / 6 over one FP32 global scale, E2M1 codes); x = bf16 (round to
    nearest even) of default_rng(1).standard_normal(2688), widened exactly to
    fp32.  Returns (codes u8[rows*cols/2], scales u8[rows*cols/16], g, x)."""
    codes, scales, g = synthetic_nvfp4(1856, 2688, seed=0)
    x = np.random.default_rng(1).standard_normal(2688, dtype=np.float32)
    return codes.reshape(-1), scales.reshape(-1), g, bf16_round(x)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 (finite input)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def dequantize(codes: np.ndarray, scales: np.ndarray, global_scale: float, rows: int,
               cols: int) -> np.ndarray:
    """float64 dequantisation (nvfp4.py:192-225 semantics, NaN scales kept)."""
    codes = np.asarray(codes, np.uint8).reshape(rows, cols // 2)
    nib = np.empty((rows, cols), np.uint8)
    nib[:, 0::2] = codes & 15
    nib[:, 1::2] = codes >> 4
    s = e4m3_table().astype(np.float64)[np.asarray(scales, np.uint8).reshape(rows, cols // GROUP)]
    return e2m1_table().astype(np.float64)[nib] * np.repeat(s, GROUP, axis=1) * float(global_scale)


# ------------------------------------------------------------- device side

def quantize_nvfp4_torch(w):
    """The same quantiser on a torch tensor (any device), for building large
    synthetic banks on the GPU.  Bit-identical to ``quantize_nvfp4`` on the
    same fp32 input."""
    import torch

    w = w.to(torch.float32).contiguous()
    rows, cols = w.shape
    dev = w.device
    blocks = w.view(rows, cols // GROUP, GROUP)
    amax = blocks.abs().amax(dim=2)
    g = (amax.max() / torch.tensor(6.0 * E4M3_MAX, dtype=torch.float32, device=dev))
    g = torch.where(g == 0, torch.ones_like(g), g)
    target = (amax / torch.tensor(6.0, dtype=torch.float32, device=dev)) / g
    t64 = torch.as_tensor(_E4M3_POS, device=dev)
    sidx = _rne_index_torch(target.to(torch.float64), t64)
    denom = t64[sidx].to(torch.float32) * g
    safe = torch.where(denom == 0, torch.ones_like(denom), denom)
    q = blocks / safe[:, :, None]
    e64 = torch.as_tensor(_E2M1_POS, device=dev)
    mag = _rne_index_torch(q.abs().to(torch.float64), e64)
    code = torch.where(denom[:, :, None] == 0, torch.zeros_like(mag), mag)
    code = torch.where((q < 0) & (code != 0), code | 8, code).to(torch.uint8).view(rows, cols)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
    return packed, sidx.to(torch.uint8).contiguous(), g


def _rne_index_torch(mag, table):
    import torch

    hi = torch.searchsorted(table, mag.contiguous(), right=False).clamp_(0, table.numel() - 1)
    lo = (hi - 1).clamp_(0, table.numel() - 1)
    d_lo = mag - table[lo]
    d_hi = table[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    idx = torch.where(pick_hi, hi, lo)
    return torch.where(mag >= table[-1], torch.full_like(idx, table.numel() - 1), idx)
