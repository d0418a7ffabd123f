"""A small, deterministic Nemotron-shaped safetensors checkpoint for the loader
tests: two shards plus ``model.safetensors.index.json`` and ``config.json``
(hybrid pattern ``ME*E``: layers 1 and 3 are MoE), NVFP4 experts (U8 codes,
F8_E4M3 group-16 scales, F32 ``weight_scale_2``), F32 router weights and BF16
/ F32 extras.  The safetensors layout is written by hand: 8-byte
little-endian header length, JSON header with ``data_offsets`` relative to
the end of the header, then the data."""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

HIDDEN, INTER, N_EXPERTS = 64, 32, 4
PATTERN = "ME*E"


def write_safetensors(path: Path, tensors: dict) -> None:
    """tensors: name -> (dtype string, shape, raw bytes)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def tensors(seed: int = 0) -> dict:
    r = np.random.default_rng(seed)
    out = {}

    def nvfp4(prefix, rows, cols):
        codes = r.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
        scales = r.integers(0, 0x7F, size=(rows, cols // 16), dtype=np.uint8)  # finite E4M3
        g = np.array([r.uniform(1e-4, 1e-2)], np.float32)
        out[f"{prefix}.weight"] = ("U8", codes.shape, codes.tobytes())
        out[f"{prefix}.weight_scale"] = ("F8_E4M3", scales.shape, scales.tobytes())
        out[f"{prefix}.weight_scale_2"] = ("F32", (), g.tobytes())

    for layer, ch in enumerate(PATTERN):
        p = f"backbone.layers.{layer}"
        if ch == "E":
            for e in range(N_EXPERTS):
                nvfp4(f"{p}.mixer.experts.{e}.up_proj", INTER, HIDDEN)
                nvfp4(f"{p}.mixer.experts.{e}.down_proj", HIDDEN, INTER)
            gw = (r.standard_normal((N_EXPERTS, HIDDEN)) * 0.1).astype(np.float32)
            gb = (r.standard_normal(N_EXPERTS) * 0.01).astype(np.float32)
            out[f"{p}.mixer.gate.weight"] = ("F32", gw.shape, gw.tobytes())
            out[f"{p}.mixer.gate.e_score_correction_bias"] = ("F32", gb.shape, gb.tobytes())
        else:
            w = (r.standard_normal((HIDDEN, HIDDEN)) * 0.02).astype(np.float32)
            bf = (w.view(np.uint32) >> 16).astype(np.uint16)
            out[f"{p}.mixer.proj.weight"] = ("BF16", bf.shape, bf.tobytes())
    return out


def write_checkpoint(root: Path, seed: int = 0) -> Path:
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    ts = tensors(seed)
    names = list(ts)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half],
              "model-00002-of-00002.safetensors": names[half:]}
    weight_map = {}
    for shard, ns in shards.items():
        write_safetensors(root / shard, {n: ts[n] for n in ns})
        weight_map.update({n: shard for n in ns})
    (root / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    (root / "config.json").write_text(json.dumps({
        "hybrid_override_pattern": PATTERN, "n_routed_experts": N_EXPERTS,
        "moe_intermediate_size": INTER, "hidden_size": HIDDEN, "num_experts_per_tok": 2}))
    return root
