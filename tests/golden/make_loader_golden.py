"""Generates tests/golden/loader_golden.json with the reference's own loader.

Builds the synthetic checkpoint of tests/ckpt_synth.py (seed 0) in a
temporary directory, opens it with kennydd001/ervf's ShardIndex
(src/moe_lab/lightningstream_nemotron/loader.py:54-185, imported from the
reference tree: $ERVF_REFERENCE, else a directory named ``reference``
beside this repository's root) and
records what it returns: sha256 of read_raw for every tensor, get_scalar of
every weight_scale_2, sha256 of dequantize_linear of every NVFP4 projection
(float32 bytes), get_float32 of the BF16 / F32 tensors, quant_kind and
layer_types.  Run once where the reference is present:

    python tests/golden/make_loader_golden.py
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
REF = Path(os.environ.get("ERVF_REFERENCE") or HERE.parents[2] / "reference")
sys.path.insert(0, str(REF / "src"))

import numpy as np  # noqa: E402

import ckpt_synth  # noqa: E402
from moe_lab.lightningstream_nemotron.loader import ShardIndex  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    with tempfile.TemporaryDirectory() as d:
        root = ckpt_synth.write_checkpoint(Path(d), seed=0)
        idx = ShardIndex(root)
        out = {"raw": {}, "scalar": {}, "dequant": {}, "float32": {}, "quant_kind": {}}
        for name in sorted(idx.entries):
            out["raw"][name] = sha(idx.read_raw(name))
            if name.endswith("weight_scale_2"):
                out["scalar"][name] = idx.get_scalar(name)
            if idx.entries[name].dtype in ("BF16", "F32") and not name.endswith("weight_scale_2"):
                out["float32"][name] = sha(idx.get_float32(name))
        prefixes = sorted({n.rsplit(".", 1)[0] for n in idx.entries if n.endswith(".weight")})
        for p in prefixes:
            out["quant_kind"][p] = idx.quant_kind(p)
            if idx.quant_kind(p) == "nvfp4":
                out["dequant"][p] = sha(idx.dequantize_linear(p))
        out["layer_types"] = list(idx.layer_types())
    (HERE / "loader_golden.json").write_text(json.dumps(out, indent=1, sort_keys=True))
    print(f"wrote {HERE / 'loader_golden.json'}: {len(out['raw'])} tensors")


if __name__ == "__main__":
    main()
