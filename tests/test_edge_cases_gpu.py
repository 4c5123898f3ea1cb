"""Edge cases of the kernels on the GPU: empty inputs (no rows, no tokens,
no sequences) return empty results without a launch error; a prefill batch
may contain a sequence with no query rows; a block-table entry outside the
pool is never accessed and is reported as device code 5, and the other
sequences' results are unchanged (the prefill kernel reads zeros in its
place; the decode kernel's result for that sequence is undefined)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as OA

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(cuda_device):
    from nanopointllm_b200 import _lib, paged_attention, runner, w8a8
    return type("K", (), dict(lib=_lib, W=w8a8, PA=paged_attention, R=runner, dev=cuda_device))


def test_empty_inputs(K):
    dev = K.dev
    x = torch.empty((0, 4096), dtype=torch.float16, device=dev)
    q, s = K.W.dynamic_per_token_quant(x)
    assert q.shape == (0, 4096) and s.shape == (0, 1)
    qw = torch.randint(-127, 128, (256, 4096), dtype=torch.int8, device=dev)
    sw = torch.rand(256, device=dev)
    out = K.W.linear_q(torch.empty((0, 4096), dtype=torch.int8, device=dev),
                       torch.empty((0,), dtype=torch.float32, device=dev), qw, sw)
    assert out.shape == (0, 256)
    kc = torch.zeros(4, 16, 2, 128, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    bt = torch.zeros(0, 2, dtype=torch.int32, device=dev)
    cl = torch.zeros(0, dtype=torch.int32, device=dev)
    o = K.PA.paged_decode_attention(torch.empty(0, 2, 128, dtype=torch.float16, device=dev), kc, vc, bt, cl,
                                    0.1, 1)
    assert o.shape == (0, 2, 128)
    o = K.PA.paged_varlen_attention(torch.empty(0, 2, 128, dtype=torch.float16, device=dev), kc, vc, bt, cl, cl,
                                    cl, 0.1, 1)
    assert o.shape == (0, 2, 128)
    torch.cuda.synchronize()
    K.lib.device_status()


def _prefill_case(seed, q_lens, ctx, H=4, Hkv=2, D=128, bs=16):
    rng = np.random.default_rng(seed)
    max_blocks = max(-(-c // bs) for c in ctx) + 1
    nb = len(ctx) * max_blocks + 2
    q_lens = np.array(q_lens, np.int32)
    return dict(q=rng.standard_normal((int(q_lens.sum()), H, D)).astype(np.float16),
                k_cache=rng.standard_normal((nb, bs, Hkv, D)).astype(np.float16),
                v_cache=rng.standard_normal((nb, bs, Hkv, D)).astype(np.float16),
                block_tables=rng.permutation(nb)[:len(ctx) * max_blocks].reshape(len(ctx), max_blocks).astype(np.int32),
                context_lens=np.array(ctx, np.int32), q_lens=q_lens,
                q_offsets=np.concatenate([[0], np.cumsum(q_lens)[:-1]]).astype(np.int32),
                scale=np.float32(D ** -0.5), groups=np.int32(H // Hkv))


def _run_prefill(K, a):
    t = {k: torch.from_numpy(np.ascontiguousarray(a[k])).to(K.dev)
         for k in ("q", "k_cache", "v_cache", "block_tables", "context_lens", "q_lens", "q_offsets")}
    o = K.PA.paged_varlen_attention(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"],
                                    t["q_lens"], t["q_offsets"], float(a["scale"]), int(a["groups"]))
    torch.cuda.synchronize()
    return o.cpu().numpy()


def _oracle(a):
    return OA.paged_varlen_attention(a["q"], a["k_cache"], a["v_cache"], a["block_tables"], a["context_lens"],
                                     a["q_lens"], a["q_offsets"], float(a["scale"]), int(a["groups"]))


def test_prefill_batch_with_an_empty_sequence(K):
    a = _prefill_case(4, [20, 0, 33], [20, 40, 60])
    got = _run_prefill(K, a)
    d = np.abs(got.astype(np.float32) - _oracle(a).astype(np.float32))
    assert d.max() <= 2e-3
    K.lib.device_status()


def test_prefill_bad_block_entry_is_skipped_and_reported(K):
    a = _prefill_case(6, [30, 25], [30, 60])
    ref = _oracle(a)
    a["block_tables"] = a["block_tables"].copy()
    a["block_tables"][1, 1] = 10_000  # outside the pool: sequence 1's keys 16..31
    got = _run_prefill(K, a)
    assert np.isfinite(got.astype(np.float32)).all()
    d = np.abs(got[:30].astype(np.float32) - ref[:30].astype(np.float32))  # sequence 0 unaffected
    assert d.max() <= 2e-3
    with pytest.raises(K.lib.NplTimeout, match="= 5"):
        K.lib.device_status()
    K.lib.device_status()  # cleared


def test_decode_bad_block_entry_is_skipped_and_reported(K):
    dev = K.dev
    g = torch.Generator().manual_seed(2)
    kc = torch.randn(12, 64, 2, 128, generator=g).half().to(dev)
    vc = torch.randn(12, 64, 2, 128, generator=g).half().to(dev)
    q = torch.randn(2, 4, 128, generator=g).half().to(dev)
    bt = torch.tensor([[0, 1, 2], [3, 10_000, 5]], dtype=torch.int32, device=dev)
    cl = torch.tensor([150, 150], dtype=torch.int32, device=dev)
    out = K.PA.paged_decode_attention(q, kc, vc, bt, cl, 128 ** -0.5, 2)
    torch.cuda.synchronize()
    good = K.PA.paged_decode_attention(q[:1].contiguous(), kc, vc, bt[:1].contiguous(), cl[:1].contiguous(),
                                       128 ** -0.5, 2)
    torch.cuda.synchronize()
    with pytest.raises(K.lib.NplTimeout, match="= 5"):
        K.lib.device_status()
    assert torch.equal(out[:1], good)  # sequence 0 unaffected
    K.lib.device_status()
