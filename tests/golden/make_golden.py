"""Generates the golden fixtures of tests/golden/ from the reference.

Run where the kennydd001/ervf tree is present ($ERVF_REFERENCE, else a
directory named ``reference`` beside this repository's root):

    python tests/golden/make_golden.py codec     # CPU: reference nvfp4.py
    python tests/golden/make_golden.py gemv      # GPU: reference CUDA kernels

``codec`` imports the reference's own numpy codec module (no CuPy needed) and
stores its decode tables and one dequantisation.  ``gemv`` runs the
reference's CUDA kernels (oracle/_ref/libervf_ref.so, built by
oracle/build_ref.py) on seeded inputs and stores inputs' seeds and outputs;
it needs a GPU but not the reference tree.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF = Path(os.environ.get("ERVF_REFERENCE") or ROOT.parent / "reference")


def codec():
    path = REF / "src/moe_lab/lightningstream_nemotron/nvfp4.py"
    spec = importlib.util.spec_from_file_location("ref_nvfp4", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    r = np.random.default_rng(20261201)
    codes = r.integers(0, 256, 512, dtype=np.uint8)
    scales = r.integers(0, 126, 64, dtype=np.uint8)
    g = np.float32(0.0123)
    out = mod.dequantize(codes, scales, float(g))
    np.savez_compressed(HERE / "codec_tables.npz", e2m1=mod.E2M1_TABLE, e4m3=mod.E4M3_TABLE,
                        dq_codes=codes, dq_scales=scales, dq_g=g, dq_out=out)


GEMV_CASES = [  # (rows, cols, seed, regime, relu2, width, full-range scale bytes)
    (64, 2688, 1, "random", 0, 16, 0), (64, 2688, 2, "adversarial", 1, 16, 0),
    (48, 1856, 3, "zero_heavy", 0, 16, 0), (40, 2048, 4, "dense", 1, 4, 0),
    (40, 768, 5, "random", 0, 8, 0), (33, 2688, 6, "random", 1, 32, 0),
    (16, 4096, 7, "adversarial", 0, 256, 0),
    (64, 2688, 8, "random", 0, 16, 1), (48, 1856, 9, "adversarial", 1, 16, 1),
    (40, 3712, 10, "random", 0, 4, 1), (33, 768, 11, "zero_heavy", 1, 32, 1),
    (24, 2688, 12, "dense", 0, 256, 1),
]

# BASELINE config 0 (ervf_b200.formats.config0_inputs) through the reference
# ERVF-16 kernel, plain and relu^2, and through the legacy 256-thread kernel
CONFIG0_CASES = [("config0_w16", 16, 0), ("config0_w16_relu2", 16, 1), ("config0_legacy", 256, 0)]


def case_inputs(i):
    rows, cols, seed, regime, relu2, width, full = GEMV_CASES[i]
    sys.path.insert(0, str(ROOT / "tests"))
    from conftest import random_nvfp4, x_regime

    if full:
        codes, scales, g = random_nvfp4(rows, cols, seed, full_range=True)
    else:
        codes, scales, g = random_nvfp4(rows, cols, seed, nan_scales=True)
    return codes, scales, g, x_regime(cols, regime, seed)


def gemv():
    import torch

    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "oracle"))
    sys.path.insert(0, str(ROOT))
    import ref
    from ervf_b200.formats import config0_inputs, e2m1_table, e4m3_device_table

    dev = torch.device("cuda")
    e2m1 = torch.from_numpy(e2m1_table()).to(dev)
    e4m3 = torch.from_numpy(e4m3_device_table()).to(dev)

    def run(codes, scales, x, g, rows, cols, relu2, width):
        c, s, xd = (torch.from_numpy(a).to(dev) for a in (codes, scales, x))
        out = torch.zeros(rows, device=dev)
        ref.call(ref.ervf_fn(width), c.data_ptr(), s.data_ptr(), e2m1.data_ptr(), e4m3.data_ptr(),
                 xd.data_ptr(), out.data_ptr(), float(g), rows, cols, relu2, 1.0, 0)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    outs = {}
    for i, (rows, cols, seed, regime, relu2, width, full) in enumerate(GEMV_CASES):
        codes, scales, g, x = case_inputs(i)
        outs[f"case{i}"] = run(codes, scales, x, g, rows, cols, relu2, width)
    codes, scales, g, x = config0_inputs()
    for key, width, relu2 in CONFIG0_CASES:
        outs[key] = run(codes, scales, x, g, 1856, 2688, relu2, width)
    dst = Path(os.environ.get("GOLDEN_OUT", HERE))
    np.savez_compressed(dst / "gemv_reference.npz", **outs)


if __name__ == "__main__":
    {"codec": codec, "gemv": gemv}[sys.argv[1]]()
