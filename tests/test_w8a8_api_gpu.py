"""The reference's W8A8 contract functions under their own names and
signatures (nanopointllm/compression/w8a8.py:33-139), run on the GPU through
the C ABI, against the reference's outputs (tests/golden/static_linear.npz,
kat.npz) and the numpy oracle. Everything here is integer or a fixed
sequence of fp32 roundings, so every comparison is exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import w8a8 as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W(cuda_device):
    from nanopointllm_b200 import w8a8
    return w8a8


def cpu(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _case(tag, dev):
    from nanopointllm_b200 import synthetic as S
    g = golden("static_linear.npz")
    m, k, n, seed = (int(v) for v in g[f"{tag}_shape"])
    dtype = torch.float16 if tag.endswith("f16") else torch.float32
    x, w = (t.to(dtype).to(dev) for t in S.config1_inputs(seed=seed, m=m, k=k, n=n))
    return g, x, w


@pytest.mark.parametrize("tag", ["tensor_f16", "tensor_f32"])
def test_static_tensor_scale_linear_matches_reference(W, cuda_device, tag):
    g, x, w = _case(tag, cuda_device)
    bias = torch.from_numpy(g[f"{tag}_bias"]).to(cuda_device)
    s = W.static_activation_scale(x.float().abs().max())
    np.testing.assert_array_equal(cpu(s), g[f"{tag}_s_tensor"])
    np.testing.assert_array_equal(cpu(W.quantize_symmetric(x, s)), g[f"{tag}_qa"])
    out, acc = W.integer_linear_per_output_reference(x, w, activation_scale=s, bias=bias)
    np.testing.assert_array_equal(cpu(acc), g[f"{tag}_acc"])
    np.testing.assert_array_equal(cpu(out), g[f"{tag}_out"])
    qdq = W.static_activation_qdq(x, s)
    assert qdq.dtype == x.dtype
    np.testing.assert_array_equal(cpu(qdq), g[f"{tag}_x_static_qdq"])
    # the module form with the same static scale: its fp32 output is the golden's
    lin = W.W8A8Linear.from_float(w, bias, activation_scale=s)
    np.testing.assert_array_equal(cpu(lin(x.float())), g[f"{tag}_out"])


@pytest.mark.parametrize("tag", ["tensor_f16", "tensor_f32"])
def test_given_per_token_scale_linear_matches_reference(W, cuda_device, tag):
    """Per-token scales the caller computed itself (fp32, not fp16 values)."""
    g, x, w = _case(tag, cuda_device)
    bias = torch.from_numpy(g[f"{tag}_bias"]).to(cuda_device)
    s_tok = torch.from_numpy(g[f"{tag}_s_tok"]).to(cuda_device)
    out, acc = W.integer_linear_per_output_reference(x, w, activation_scale=s_tok, bias=bias)
    np.testing.assert_array_equal(cpu(acc), g[f"{tag}_acc_tok"])
    np.testing.assert_array_equal(cpu(out), g[f"{tag}_out_tok"])
    out2, acc2 = W.integer_linear_per_output(x, w, activation_scale=s_tok, bias=bias)
    assert torch.equal(out, out2) and torch.equal(acc, acc2)


@pytest.mark.parametrize("tag", ["tensor_f16", "tensor_f32"])
def test_qdq_functions_match_reference(W, cuda_device, tag):
    g, x, w = _case(tag, cuda_device)
    w_deq, qw, ws = W.per_output_weight_qdq(w)
    assert w_deq.dtype == w.dtype and qw.dtype == torch.int8 and qw.shape == w.shape
    np.testing.assert_array_equal(cpu(qw), g[f"{tag}_qw"])
    np.testing.assert_array_equal(cpu(ws), g[f"{tag}_ws"])
    np.testing.assert_array_equal(cpu(w_deq), g[f"{tag}_w_deq"])
    x_qdq, x_s = W.dynamic_per_token_activation_qdq(x)
    assert x_qdq.dtype == x.dtype and x_s.shape == (x.shape[0], 1)
    np.testing.assert_array_equal(cpu(x_qdq), g[f"{tag}_x_dyn_qdq"])
    np.testing.assert_array_equal(cpu(x_s), g[f"{tag}_x_dyn_s"])


def test_linear_kat_static_scale(W, cuda_device):
    """tests/test_w8a8_contract.py:55-76 of the reference: K = 4 (not a
    multiple of 16: zero columns are appended on the device), static scale,
    bias."""
    kat = golden("kat.npz")
    x, w, b = (torch.from_numpy(kat[n]).to(cuda_device) for n in ("lin_x", "lin_w", "lin_b"))
    s = W.static_activation_scale(x.abs().max())
    np.testing.assert_array_equal(cpu(s), kat["lin_s"])
    out, acc = W.integer_linear_per_output_reference(x, w, activation_scale=s, bias=b)
    np.testing.assert_array_equal(cpu(acc), kat["lin_acc"])
    np.testing.assert_array_equal(cpu(out), kat["lin_out"])
    q = W.quantize_symmetric(torch.from_numpy(kat["quant_in"]).to(cuda_device), 1.0)
    np.testing.assert_array_equal(cpu(q), kat["quant_out"])


def test_scale_from_absmax_edges(W, cuda_device):
    a = np.array([0.0, 1e-30, 2.0 ** -14, 6e-5, 0.5, 1.0, 127.0, 1234.5, 65504.0, 1e6], np.float32)
    got = W.scale_from_absmax(torch.from_numpy(a).to(cuda_device))
    np.testing.assert_array_equal(cpu(got), O.scale_from_absmax(a))


@pytest.mark.parametrize("k", [40, 100, 4096])
def test_ragged_k_and_axis(W, cuda_device, k):
    gen = torch.Generator().manual_seed(k)
    x = (torch.randn(3, 7, k, generator=gen) * 4).half()
    w = (torch.randn(33, k, generator=gen) * 0.02).half()
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    out, acc = W.integer_linear_per_output(xd, wd)
    s = O.scale_from_absmax(np.abs(x.float().numpy()).max(-1, keepdims=True))
    oo, oa = O.integer_linear_per_output_reference(x.numpy(), w.numpy(), activation_scale=s)
    np.testing.assert_array_equal(cpu(acc), oa)
    np.testing.assert_array_equal(cpu(out), oo)
    # axis 1: one scale per (batch, column) slice along the 7 tokens
    qdq, sc = W.dynamic_per_token_activation_qdq(xd, axis=1)
    xt = np.moveaxis(x.numpy(), 1, -1)
    qa, sa = O.dynamic_per_token_quant(xt)
    np.testing.assert_array_equal(cpu(sc), np.moveaxis(sa, -1, 1))
    np.testing.assert_array_equal(cpu(qdq), np.moveaxis((qa.astype(np.float32) * sa).astype(np.float16), -1, 1))


def test_nonpositive_scale_raises(W, cuda_device):
    x = torch.ones(2, 16, device=cuda_device)
    with pytest.raises(ValueError, match="positive"):
        W.quantize_symmetric(x, torch.tensor([[1.0], [0.0]], device=cuda_device))
    with pytest.raises(ValueError, match="positive"):
        W.integer_linear_per_output_reference(x, torch.ones(4, 16, device=cuda_device), activation_scale=-1.0)
    with pytest.raises(ValueError, match="shapes"):
        W.integer_linear_per_output_reference(x, torch.ones(4, 8, device=cuda_device), activation_scale=1.0)
