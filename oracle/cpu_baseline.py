"""CPU baseline: torch FP32 dequant-then-matmul of the routed-expert block.

TEST / BASELINE INFRASTRUCTURE, used only by bench.py's cpu_baseline leg and
its ``--impl reference`` arm.  It restates the reference's CPU path -- numpy
dequantisation (nvfp4.dequantize, src/moe_lab/lightningstream_nemotron/
nvfp4.py:192-225) followed by the float64 module semantics
(reference.mlp_relu2 / moe_forward, reference.py:119-154) -- in FP32 torch on
the host cores, as the build's baseline plan asks: dequantise with the device
tables (E4M3 NaN -> 0), then ``torch.matmul``.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


def _e4m3_table() -> torch.Tensor:
    t = np.zeros(256, np.float32)
    for b in range(256):
        e, m = (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            v = 0.0
        elif e == 0:
            v = (m / 8.0) * 2.0 ** -6
        else:
            v = (1 + m / 8.0) * 2.0 ** (e - 7)
        t[b] = -v if b & 0x80 else v
    return torch.from_numpy(t)


_E4M3 = _e4m3_table()


def use_all_cores() -> int:
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def dequant(codes: torch.Tensor, scales: torch.Tensor, g: float, rows: int, cols: int) -> torch.Tensor:
    """u8 codes [rows*cols/2] + E4M3 scales [rows*cols/16] -> fp32 [rows, cols]."""
    c = codes.view(rows, cols // 2)
    nib = torch.stack((c & 15, c >> 4), dim=2).view(rows, cols).long()
    s = _E4M3[scales.view(rows, cols // 16).long()] * torch.tensor(g, dtype=torch.float32)
    return _E2M1[nib] * s.repeat_interleave(16, dim=1)


def moe_layer(x: torch.Tensor, experts, ids, weights, hidden: int, inter: int) -> torch.Tensor:
    """x + sum_s w_s * down_s(relu(up_s(x))^2), dequant-then-matmul per expert."""
    out = x.clone()
    for s, e in enumerate(ids):
        (uc, us, ug), (dc, ds, dg) = experts[int(e)]
        up = dequant(uc, us, ug, inter, hidden)
        h = torch.clamp(up @ x, min=0.0) ** 2
        dn = dequant(dc, ds, dg, hidden, inter)
        out += float(weights[s]) * (dn @ h)
    return out


def moe_layer_timed(x: torch.Tensor, experts, ids, weights, hidden: int, inter: int):
    """moe_layer with the two phases timed apart: returns (out, dequant_s,
    matmul_s), the seconds spent dequantising the routed experts and in the
    matmuls (+ relu^2 and the weighted sum)."""
    out = x.clone()
    t_dq = t_mm = 0.0
    for s, e in enumerate(ids):
        (uc, us, ug), (dc, ds, dg) = experts[int(e)]
        t0 = time.perf_counter()
        up = dequant(uc, us, ug, inter, hidden)
        dn = dequant(dc, ds, dg, hidden, inter)
        t1 = time.perf_counter()
        h = torch.clamp(up @ x, min=0.0) ** 2
        out += float(weights[s]) * (dn @ h)
        t_mm += time.perf_counter() - t1
        t_dq += t1 - t0
    return out, t_dq, t_mm
