"""SiLU * up on the GPU (npl_silu_mul, and the same device function inside the
gate/up epilogue of the linear) against the oracle's fp64 SiLU rounded once
to fp16 (reference: act_fn(gate) * up, lightweight_runner.py:358).

The kernel evaluates SiLU in fp32 and falls back to fp64 only where the fp32
value lies too close to an fp16 rounding midpoint; these tests check that the
result is bit-identical to the fp64 evaluation for every fp16 input.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a8 as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W(cuda_device):
    from nanopointllm_b200 import w8a8
    return w8a8


def test_silu_every_fp16_value(W, cuda_device):
    """All 65536 fp16 bit patterns as the gate, up = 1: the output is the
    fp16 SiLU itself. Bit-exact against the oracle for every finite input
    (signed zeros included); NaN in, NaN out."""
    bits = np.arange(1 << 16, dtype=np.uint16)
    g = bits.view(np.float16).reshape(256, 256)
    u = np.ones_like(g)
    out = W.silu_mul(torch.from_numpy(g).to(cuda_device), torch.from_numpy(u).to(cuda_device)).cpu().numpy()
    with np.errstate(all="ignore"):
        ref = O.silu_mul(g, u)
    fin = np.isfinite(g.astype(np.float32)) & np.isfinite(ref.astype(np.float32))
    assert fin.sum() > 63000
    np.testing.assert_array_equal(out[fin].view(np.uint16), ref[fin].view(np.uint16))
    nan_in = np.isnan(g.astype(np.float32))
    assert np.isnan(out[nan_in].astype(np.float32)).all()
    # non-finite results where the oracle has them (silu(-inf) = nan, silu(inf) = inf)
    other = ~fin & ~nan_in
    np.testing.assert_array_equal(np.isnan(out[other].astype(np.float32)), np.isnan(ref[other].astype(np.float32)))


@pytest.mark.parametrize("rows,cols", [(8, 11008), (3, 40), (1, 8)])
def test_silu_mul_random(W, cuda_device, rows, cols):
    """Random gate/up rows at the MLP widths (fp16 products rounded once)."""
    gen = torch.Generator().manual_seed(rows * 131 + cols)
    g = (torch.randn(rows, cols, generator=gen) * 3).half()
    u = (torch.randn(rows, cols, generator=gen) * 2).half()
    out = W.silu_mul(g.to(cuda_device), u.to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint16), O.silu_mul(g.numpy(), u.numpy()).view(np.uint16))


def test_silu_mul_rejects_bad_shapes(W, cuda_device):
    g = torch.zeros(4, 16, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError):
        W.silu_mul(g, torch.zeros(4, 8, dtype=torch.float16, device=cuda_device))
    with pytest.raises(ValueError):
        W.silu_mul(g.float(), g.float())
