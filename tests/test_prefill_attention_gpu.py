"""Varlen paged prefill attention on the GPU (npl_paged_prefill_attention,
tcgen05 kind::f16) against the reference's own kernel and the numpy oracle.

The golden outputs in tests/golden/prefill_attention.npz come from the
reference's Triton kernel (paged_attention.py:1037-1139) run in Triton's CPU
interpreter (tests/golden/make_prefill_golden.py). Both the reference and
this kernel round the probabilities to fp16 for the P.V product, with
different key tiles (64 there, 128 here) and a different exp and summation
order, so the results agree to fp16 rounding: tolerance ATOL = 2e-3 on
outputs of magnitude <= ~1, plus a bound on the mean error.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import attention as OA

pytestmark = pytest.mark.gpu

ATOL = 2e-3
MEAN_ATOL = 5e-5


def _run(PA, a, dev, out=None, max_q_len=None):
    t = {k: torch.from_numpy(np.ascontiguousarray(a[k])).to(dev)
         for k in ("q", "k_cache", "v_cache", "block_tables", "context_lens", "q_lens", "q_offsets")}
    o = PA.paged_varlen_attention(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"],
                                  t["q_lens"], t["q_offsets"], float(a["scale"]), int(a["groups"]), out=out,
                                  max_q_len=max_q_len)
    torch.cuda.synchronize()
    return o.cpu().numpy()


def _close(got, want, what):
    d = np.abs(got.astype(np.float32) - want.astype(np.float32))
    assert np.isfinite(got).all(), what
    assert d.max() <= ATOL and d.mean() <= MEAN_ATOL, f"{what}: max {d.max()} mean {d.mean()}"


def _case(seqs, H, Hkv, D, bs, seed, scale_q=1.0):
    rng = np.random.default_rng(seed)
    max_blocks = max(-(-c // bs) for _, c in seqs) + 1
    nb = len(seqs) * max_blocks + 2
    q_lens = np.array([ql for ql, _ in seqs], np.int32)
    offs = np.concatenate([[0], np.cumsum(q_lens)[:-1]]).astype(np.int32)
    return dict(
        q=(rng.standard_normal((int(q_lens.sum()), H, D)) * scale_q).astype(np.float16),
        k_cache=rng.standard_normal((nb, bs, Hkv, D)).astype(np.float16),
        v_cache=rng.standard_normal((nb, bs, Hkv, D)).astype(np.float16),
        block_tables=rng.permutation(nb)[:len(seqs) * max_blocks].reshape(len(seqs), max_blocks).astype(np.int32),
        context_lens=np.array([c for _, c in seqs], np.int32), q_lens=q_lens, q_offsets=offs,
        scale=np.float32(D ** -0.5), groups=np.int32(H // Hkv))


def _oracle(a):
    return OA.paged_varlen_attention(a["q"], a["k_cache"], a["v_cache"], a["block_tables"], a["context_lens"],
                                     a["q_lens"], a["q_offsets"], float(a["scale"]), int(a["groups"]))


def test_reference_golden(cuda_device):
    from nanopointllm_b200 import _lib, paged_attention as PA
    g = golden("prefill_attention.npz")
    for c in g["cases"]:
        a = {k.split("__", 1)[1]: g[k] for k in g.files if k.startswith(str(c) + "__")}
        _close(_run(PA, a, cuda_device), a["out"], str(c))
    _lib.device_status()


@pytest.mark.parametrize("seqs,H,Hkv,D,bs", [
    ([(300, 300), (129, 700), (2, 2)], 8, 2, 128, 16),
    ([(560, 560)] * 2, 4, 4, 128, 256),
    ([(255, 1000), (128, 128), (7, 260)], 4, 1, 64, 32),
    ([(1, 513), (384, 384)], 2, 2, 128, 48),
])
def test_vs_oracle(cuda_device, seqs, H, Hkv, D, bs):
    from nanopointllm_b200 import _lib, paged_attention as PA
    a = _case(seqs, H, Hkv, D, bs, seed=len(seqs) * 31 + bs)
    _close(_run(PA, a, cuda_device), _oracle(a), f"{seqs} D={D} bs={bs}")
    _lib.device_status()


def test_peaked_scores_vs_oracle(cuda_device):
    """Large scores (q x 8): the running max moves often and most p round to 0."""
    from nanopointllm_b200 import paged_attention as PA
    a = _case([(200, 450)], 4, 2, 128, 16, seed=9, scale_q=8.0)
    _close(_run(PA, a, cuda_device), _oracle(a), "peaked")


def test_rows_of_no_sequence_untouched_and_status_clean(cuda_device):
    """Only the listed rows are written (a gap between two sequences keeps its
    sentinel), and valid metadata leaves the device status clear."""
    from nanopointllm_b200 import _lib, paged_attention as PA
    a = _case([(40, 90), (17, 17)], 4, 2, 128, 16, seed=3)
    q = a["q"]
    gap = 9
    q2 = np.concatenate([q[:40], np.zeros((gap, *q.shape[1:]), np.float16), q[40:]])
    b = dict(a, q=q2, q_offsets=np.array([0, 40 + gap], np.int32))
    out = torch.full(q2.shape, float("nan"), dtype=torch.float16, device=cuda_device)
    got = _run(PA, b, cuda_device, out=out, max_q_len=40)
    assert np.isnan(got[40:40 + gap].astype(np.float32)).all()
    ref = _oracle(a)
    _close(got[:40], ref[:40], "seq 0")
    _close(got[40 + gap:], ref[40:], "seq 1")
    _lib.device_status()


def test_against_fp32_sdpa(cuda_device):
    """Sanity against an fp32 PyTorch reference of the same attention
    (no fp16 rounding of the probabilities): within 4e-3."""
    import torch.nn.functional as F
    from nanopointllm_b200 import paged_attention as PA
    seqs = [(150, 400), (64, 64)]
    a = _case(seqs, 4, 2, 128, 16, seed=5)
    got = _run(PA, a, cuda_device)
    off = 0
    for b, (ql, ctx) in enumerate(seqs):
        bt = a["block_tables"][b]
        keys = np.arange(ctx)
        k = torch.from_numpy(a["k_cache"][bt[keys // 16], keys % 16]).float()
        v = torch.from_numpy(a["v_cache"][bt[keys // 16], keys % 16]).float()
        qi = torch.from_numpy(a["q"][off:off + ql]).float().permute(1, 0, 2)[None]
        ki = k.permute(1, 0, 2)[None].repeat_interleave(2, 1)
        vi = v.permute(1, 0, 2)[None].repeat_interleave(2, 1)
        allowed = torch.arange(ctx)[None, :] <= (ctx - ql) + torch.arange(ql)[:, None]
        o = F.scaled_dot_product_attention(qi, ki, vi, attn_mask=allowed, scale=float(a["scale"]))
        d = np.abs(got[off:off + ql].astype(np.float32) - o[0].permute(1, 0, 2).numpy())
        assert d.max() < 4e-3, d.max()
        off += ql


def test_argument_errors(cuda_device):
    from nanopointllm_b200 import _lib, paged_attention as PA
    a = _case([(20, 20)], 2, 2, 128, 16, seed=1)
    t = {k: torch.from_numpy(np.ascontiguousarray(a[k])).to(cuda_device) for k in a if k not in ("scale", "groups")}
    with pytest.raises(ValueError):
        PA.paged_varlen_attention(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"],
                                  t["q_lens"], t["q_offsets"], 0.1, 3)  # geometry mismatch
    with pytest.raises(_lib.NplError):
        PA.paged_varlen_attention(t["q"][..., :96].contiguous(), t["k_cache"][..., :96].contiguous(),
                                  t["v_cache"][..., :96].contiguous(), t["block_tables"], t["context_lens"],
                                  t["q_lens"], t["q_offsets"], 0.1, 1)  # head_dim 96 unsupported
