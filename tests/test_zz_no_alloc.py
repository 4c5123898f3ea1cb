"""npl_w8a8_linear_noalloc: the W8A8 linear for callers that cannot allocate
device memory (a plugin handed only its input/output buffers by a host engine
that owns the GPU memory, a binding without a CUDA allocator, a loop that must
not call cudaMalloc). Its scratch is a fixed array inside the library instead
of a caller workspace; its results must equal npl_w8a8_linear's bit for bit
(the linear tests' tolerance is exact equality), on consecutive calls that
reuse that array.

This file is collected last on purpose: it must pass both alone in a fresh
process and after every other GPU test.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(lib, qa, sa, qw, sw, out, acc, epilogue=0, residual=None, m=None):
    from nanopointllm_b200 import _lib as L
    m = qa.shape[0] if m is None else m
    n, k = qw.shape
    return lib.npl_w8a8_linear_noalloc(
        qa.data_ptr(), qa.stride(0), sa.data_ptr(), qw.data_ptr(), qw.stride(0), sw.data_ptr(), None, m, n, k,
        epilogue, None if residual is None else residual.data_ptr(), 0 if residual is None else residual.stride(0),
        out.data_ptr(), out.stride(0), L.NPL_F16, None if acc is None else acc.data_ptr(),
        L.stream_ptr(qa.device))


@pytest.mark.parametrize("m,n,k,epilogue", [(8, 12288, 4096, 0), (64, 4096, 11008, 1), (3, 1000, 512, 0)])
def test_noalloc_matches_workspace_linear_twice(cuda_device, m, n, k, epilogue):
    from nanopointllm_b200 import _lib as L
    from nanopointllm_b200 import w8a8 as W
    dev = cuda_device
    gen = torch.Generator().manual_seed(m + n + k)
    qa = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8).to(dev)
    qw = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8).to(dev)
    sa = (torch.rand(m, generator=gen) * 0.05 + 0.001).to(dev)
    sw = (torch.rand(n, generator=gen) * 0.001 + 1e-5).to(dev)
    res = torch.randn(m, n, generator=gen).half().to(dev) if epilogue == L.EPI_RESIDUAL else None
    ref_acc = torch.empty((m, n), dtype=torch.int32, device=dev)
    ref = W.linear_q(qa, sa, qw, sw, epilogue=epilogue, residual=res, acc_out=ref_acc)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        out = torch.empty_like(ref)
        acc = torch.empty_like(ref_acc)
        L.check(_noalloc(L.lib, qa, sa, qw, sw, out, acc, epilogue=epilogue, residual=res))
        torch.cuda.synchronize()
        assert torch.equal(acc, ref_acc)
        assert torch.equal(out, ref)
    L.device_status()


def test_noalloc_rejects_more_tokens_than_its_scratch(cuda_device):
    from nanopointllm_b200 import _lib as L
    dev = cuda_device
    m, n, k = 65, 256, 256
    qa = torch.zeros((m, k), dtype=torch.int8, device=dev)
    qw = torch.zeros((n, k), dtype=torch.int8, device=dev)
    sa = torch.ones(m, device=dev)
    sw = torch.ones(n, device=dev)
    out = torch.empty((m, n), dtype=torch.float16, device=dev)
    rc = _noalloc(L.lib, qa, sa, qw, sw, out, None)
    assert rc == L.NPL_ERR_ARG
    assert b"at most 64" in L.lib.npl_last_error_string()
