"""Host-side layout of the packed gate/up weight (w8a8.pack_gate_up), which
the SiLU * up epilogue of the linear kernel depends on: groups of 16 rows,
8 gate rows followed by the same 8 output rows of up, so that a 128-row
weight tile holds the gate and up rows of 64 outputs and TMEM lanes l and
l + 8 of every 16-lane group are a gate row and its up row."""
from __future__ import annotations

import pytest
import torch


@pytest.fixture(scope="module")
def W():
    from nanopointllm_b200 import w8a8
    return w8a8


def test_rows_interleaved_by_eight(W):
    inter, k = 128, 3
    gate = torch.arange(inter * k, dtype=torch.int32).reshape(inter, k)
    up = -gate - 1
    p = W.pack_gate_up(gate, up)
    assert p.shape == (2 * inter, k)
    for r in range(2 * inter):
        grp, i = divmod(r, 16)
        src = gate if i < 8 else up
        assert torch.equal(p[r], src[8 * grp + i % 8])


def test_scales_and_tiles(W):
    """Per-row scales pack like the weight rows; 128-row tile t holds the
    gate and up rows of outputs [64 t, 64 t + 64)."""
    inter = 192
    gs = torch.arange(inter, dtype=torch.float32)
    us = 1000 + gs
    p = W.pack_gate_up(gs, us)
    for t in range(2 * inter // 128):
        tile = p[128 * t:128 * (t + 1)]
        assert set(tile[tile < 1000].tolist()) == set(range(64 * t, 64 * t + 64))
        assert set((tile[tile >= 1000] - 1000).tolist()) == set(range(64 * t, 64 * t + 64))


def test_rejects_ragged_or_mismatched(W):
    with pytest.raises(ValueError):
        W.pack_gate_up(torch.zeros(100, 4), torch.zeros(100, 4))
    with pytest.raises(ValueError):
        W.pack_gate_up(torch.zeros(128, 4), torch.zeros(64, 4))
