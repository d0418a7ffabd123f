"""Checkpoint ingestion (ervf_b200.loader) on a synthetic safetensors
checkpoint: the index reads what the reference's ShardIndex reads (golden
fixture made with the reference loader, tests/golden/make_loader_golden.py),
the bank holds every expert record at its slot, the router tensors load, and
bad checkpoints are rejected.  The GPU test streams the bank into HBM through
the pinned staging ring and decodes with it."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import ckpt_synth

GOLDEN = Path(__file__).resolve().parent / "golden" / "loader_golden.json"


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    return ckpt_synth.write_checkpoint(tmp_path_factory.mktemp("ckpt"), seed=0)


def test_index_matches_reference_loader(ckpt):
    from ervf_b200.loader import ShardIndex

    gold = json.loads(GOLDEN.read_text())
    idx = ShardIndex(ckpt)
    assert sorted(idx.entries) == sorted(gold["raw"])
    for name, h in gold["raw"].items():
        assert _sha(idx.read_raw(name)) == h, name
    for name, v in gold["scalar"].items():
        assert idx.get_scalar(name) == v, name
    for name, h in gold["float32"].items():
        assert _sha(idx.get_float32(name)) == h, name
    for prefix, kind in gold["quant_kind"].items():
        assert idx.quant_kind(prefix) == kind, prefix
    for prefix, h in gold["dequant"].items():
        assert _sha(idx.dequantize_linear(prefix)) == h, prefix
    assert list(idx.layer_types()) == gold["layer_types"]
    assert idx.moe_layers() == [1, 3]
    idx.close()


def test_bank_holds_every_record(ckpt):
    from ervf_b200.loader import ShardIndex, expert_prefix, load_expert_bank

    idx = ShardIndex(ckpt)
    bank = load_expert_bank(idx, device="cpu", staging_bytes=1000)
    H, I, E = ckpt_synth.HIDDEN, ckpt_synth.INTER, ckpt_synth.N_EXPERTS
    assert (bank.n_layers, bank.n_experts, bank.hidden, bank.inter) == (2, E, H, I)
    assert bank.checkpoint_layers == [1, 3]
    for l, layer in enumerate((1, 3)):
        for e in range(E):
            pre = expert_prefix(layer, e)
            (uc, us, ug), (dc, ds, dg) = bank.expert_host(l, e)
            assert np.array_equal(uc, idx.read_raw(f"{pre}.up_proj.weight"))
            assert np.array_equal(us, idx.read_raw(f"{pre}.up_proj.weight_scale"))
            assert np.array_equal(dc, idx.read_raw(f"{pre}.down_proj.weight"))
            assert np.array_equal(ds, idx.read_raw(f"{pre}.down_proj.weight_scale"))
            assert ug == np.float32(idx.get_scalar(f"{pre}.up_proj.weight_scale_2"))
            assert dg == np.float32(idx.get_scalar(f"{pre}.down_proj.weight_scale_2"))
    idx.close()


def test_router_tensors(ckpt):
    from ervf_b200.loader import ShardIndex, load_router

    idx = ShardIndex(ckpt)
    gw, gb = load_router(idx, device="cpu")
    assert gw.shape == (2, ckpt_synth.N_EXPERTS, ckpt_synth.HIDDEN)
    assert np.array_equal(gw[1].numpy(), idx.get_float32("backbone.layers.3.mixer.gate.weight"))
    assert np.array_equal(gb[0].numpy(),
                          idx.get_float32("backbone.layers.1.mixer.gate.e_score_correction_bias"))


def test_rejects_inconsistent_records(tmp_path):
    from ervf_b200.loader import ShardIndex, load_expert_bank

    ts = ckpt_synth.tensors(1)
    name = "backbone.layers.3.mixer.experts.2.up_proj.weight_scale"
    dtype, shape, raw = ts[name]
    ts[name] = (dtype, (shape[0], shape[1] - 1), raw[: shape[0] * (shape[1] - 1)])
    ckpt_synth.write_safetensors(tmp_path / "model.safetensors", ts)
    (tmp_path / "config.json").write_text(json.dumps({"hybrid_override_pattern": "ME*E"}))
    idx = ShardIndex(tmp_path)
    with pytest.raises(ValueError):
        load_expert_bank(idx, device="cpu")
    with pytest.raises(ValueError):
        idx.dequantize_linear("backbone.layers.3.mixer.experts.2.up_proj")


@pytest.mark.gpu
def test_gpu_bank_streams_and_decodes(ckpt, cuda):
    """The pinned-staging upload gives the same bank as per-expert uploads;
    a decode step on it equals the step on the directly uploaded bank."""
    from ervf_b200.loader import ShardIndex, load_expert_bank, load_router
    from ervf_b200.moe import ExpertBank, MoEDecoder

    idx = ShardIndex(ckpt)
    bank = load_expert_bank(idx, device=cuda, staging_bytes=4096, depth=2)
    ref = ExpertBank(bank.n_layers, bank.n_experts, bank.hidden, bank.inter, cuda)
    for l in range(bank.n_layers):
        for e in range(bank.n_experts):
            up, dn = bank.expert_host(l, e)
            ref.upload_expert(l, e, up, dn)
        assert torch.equal(bank.up_codes[l], ref.up_codes[l])
        assert torch.equal(bank.dn_scales[l], ref.dn_scales[l])
        assert torch.equal(bank.globals[l], ref.globals[l])
    gw, gb = load_router(idx, device=cuda)
    x = torch.randn(bank.hidden, device=cuda)
    k = 2
    y1 = MoEDecoder(bank, k).step_with_router(x, gw, gb).clone()
    y2 = MoEDecoder(ref, k).step_with_router(x, gw, gb).clone()
    torch.cuda.synchronize()
    assert torch.isfinite(y1).all()
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))
