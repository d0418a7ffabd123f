"""Host-side helpers of bench.py (no GPU): the busiest-rank record count that
the expert-parallel roofline fraction of the batch-1 line uses."""

from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402


def test_busiest_rank_slots_one_rank_is_every_slot():
    g = torch.Generator().manual_seed(3)
    rl = torch.randn(5, 24, 128, generator=g)
    got = bench.busiest_rank_slots(rl, 1, 6)
    assert got.shape == (5,) and torch.all(got == 24 * 6)


def test_busiest_rank_slots_counts_the_most_loaded_owner():
    rl = torch.full((1, 2, 16), -10.0)
    # layer 0: experts 0, 2, 4, 1 -> ranks 0, 0, 0, 1 with 2 ranks: busiest 3
    for e, v in ((0, 4.0), (2, 3.0), (4, 2.0), (1, 1.0)):
        rl[0, 0, e] = v
    # layer 1: experts 1, 3, 5, 7 -> all rank 1 of 2: busiest 4
    for e, v in ((1, 4.0), (3, 3.0), (5, 2.0), (7, 1.0)):
        rl[0, 1, e] = v
    assert bench.busiest_rank_slots(rl, 2, 4).tolist() == [7.0]
    # 4 ranks: layer 0 -> ranks 0, 2, 0, 1 (2); layer 1 -> ranks 1, 3, 1, 3 (2)
    assert bench.busiest_rank_slots(rl, 4, 4).tolist() == [4.0]


def test_busiest_rank_slots_bounds():
    g = torch.Generator().manual_seed(5)
    rl = torch.randn(64, 24, 128, generator=g)
    for world in (2, 4, 8):
        b = bench.busiest_rank_slots(rl, world, 6)
        assert torch.all(b >= 24 * 6 / world) and torch.all(b <= 24 * 6)
