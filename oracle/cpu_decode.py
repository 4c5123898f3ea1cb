"""The reference's CPU W8A8 decode path, restated in torch on the host cores.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the timed CPU baseline of
bench.py (its ``cpu_baseline`` leg and ``--impl reference``), never the
product path.

The reference has no int8 GPU path; its W8A8 decode is the eager runner with
every Linear evaluated by the CPU integer golden. One decoder layer of that
path at the 7B geometry, with the reference's own torch CPU arithmetic:

* RMSNorm, eager (lightweight_runner.py:239-245): fp32 normalise, fp16, weight
  multiply in fp16;
* per-token dynamic int8 activations (compression/w8a8.py:106-115 through
  :33-50): absmax, fp16-stored scale, ``round(v / s)`` clamped to +-127;
* every Linear as integer_linear_per_output_reference (w8a8.py:118-139):
  int8 activations and int8 weights cast to int32 on every call, an int32
  matmul, then ``(acc * s_a) * s_w`` in fp32 (weights are quantised once up
  front here; the golden function re-quantises them on every call, which
  would only add to its time);
* RoPE on q and k (HF apply_rotary_pos_emb in fp16, paged_attention.py:1286-1292);
* decode attention per sequence as _paged_decode_attention_pytorch
  (paged_attention.py:846-869: the pool gathered through the block table,
  then scaled_dot_product_attention), in fp32 on the CPU;
* fp16 residual adds, SiLU(gate) * up (lightweight_runner.py:358), down.

The LM head is the same integer golden over [batch, 4096] x [32003, 4096].
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

HIDDEN, INTER, HEADS, HEAD_DIM, VOCAB = 4096, 11008, 32, 128, 32003


def _scale_from_absmax(absmax: torch.Tensor) -> torch.Tensor:
    tiny = torch.finfo(torch.float16).tiny
    return (absmax.float().clamp_min(tiny) / 127).to(torch.float16).float().clamp_min(tiny)


def _quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    s = _scale_from_absmax(x.float().abs().amax(-1, keepdim=True))
    return torch.round(x.float() / s).clamp(-127, 127).to(torch.int8), s


def _int_linear(x16: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    qa, sa = _quant_rows(x16)
    acc = qa.to(torch.int32) @ qw.to(torch.int32).transpose(0, 1)
    out = acc.float()
    out *= sa
    out *= sw.unsqueeze(0)
    return out.to(torch.float16)


def _rmsnorm(x16: torch.Tensor, w16: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x16.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.float16)
    return w16 * y


def _rope(x16: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x16.shape[-1] // 2
    rot = torch.cat((-x16[..., half:], x16[..., :half]), dim=-1)
    return x16 * cos + rot * sin


class CpuDecodeLayer:
    """One 7B-geometry decoder layer (random int8 weights, fixed scales) over a
    paged fp16 KV pool of ``batch`` sequences of ``ctx`` tokens, block 256."""

    def __init__(self, batch: int = 8, ctx: int = 1024, block_size: int = 256, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        q8 = lambda n, k: torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        sc = lambda n: torch.full((n,), 0.02 / 73.3, dtype=torch.float32)  # uniform int8 std ~73.3
        self.batch, self.ctx, self.block_size = batch, ctx, block_size
        self.w = {"qkv": (q8(3 * HIDDEN, HIDDEN), sc(3 * HIDDEN)), "o": (q8(HIDDEN, HIDDEN), sc(HIDDEN)),
                  "gate_up": (q8(2 * INTER, HIDDEN), sc(2 * INTER)), "down": (q8(HIDDEN, INTER), sc(HIDDEN))}
        self.head = (q8(VOCAB, HIDDEN), sc(VOCAB))
        self.norm = torch.ones(HIDDEN, dtype=torch.float16)
        nblk = -(-(ctx + 1) // block_size)
        self.k_cache = torch.randn(batch * nblk, block_size, HEADS, HEAD_DIM, generator=g).half()
        self.v_cache = torch.randn(batch * nblk, block_size, HEADS, HEAD_DIM, generator=g).half()
        self.block_tables = torch.randperm(batch * nblk, generator=g).reshape(batch, nblk)
        self.x = torch.randn(batch, HIDDEN, generator=g).half()
        ang = torch.arange(HEAD_DIM // 2).float()
        ang = ctx * 10000.0 ** (-2 * ang / HEAD_DIM)
        self.cos = torch.cat((ang.cos(), ang.cos())).half()
        self.sin = torch.cat((ang.sin(), ang.sin())).half()

    def _attention(self, q: torch.Tensor) -> torch.Tensor:
        n = self.ctx + 1
        outs = []
        for b in range(self.batch):
            bt = self.block_tables[b, :-(-n // self.block_size)]
            k = self.k_cache[bt].reshape(-1, HEADS, HEAD_DIM)[:n].permute(1, 0, 2).unsqueeze(0).float()
            v = self.v_cache[bt].reshape(-1, HEADS, HEAD_DIM)[:n].permute(1, 0, 2).unsqueeze(0).float()
            o = F.scaled_dot_product_attention(q[b].unsqueeze(0).unsqueeze(2).float(), k, v,
                                               scale=HEAD_DIM ** -0.5)
            outs.append(o.squeeze(0).squeeze(1))
        return torch.stack(outs).to(torch.float16)

    @torch.inference_mode()
    def layer(self, h: torch.Tensor) -> torch.Tensor:
        b = self.batch
        qkv = _int_linear(_rmsnorm(h, self.norm), *self.w["qkv"])
        q = _rope(qkv[:, :HIDDEN].reshape(b, HEADS, HEAD_DIM), self.cos, self.sin)
        k = _rope(qkv[:, HIDDEN:2 * HIDDEN].reshape(b, HEADS, HEAD_DIM), self.cos, self.sin)
        v = qkv[:, 2 * HIDDEN:].reshape(b, HEADS, HEAD_DIM)
        pos = self.ctx
        for i in range(b):  # store_kvcache of the new token (paged_attention.py:386-401)
            blk = int(self.block_tables[i, pos // self.block_size])
            self.k_cache[blk, pos % self.block_size] = k[i]
            self.v_cache[blk, pos % self.block_size] = v[i]
        a = self._attention(q).reshape(b, HIDDEN)
        h = h + _int_linear(a, *self.w["o"])
        gu = _int_linear(_rmsnorm(h, self.norm), *self.w["gate_up"])
        act = F.silu(gu[:, :INTER]) * gu[:, INTER:]
        return h + _int_linear(act, *self.w["down"])

    @torch.inference_mode()
    def lm_head(self, h: torch.Tensor) -> torch.Tensor:
        return _int_linear(_rmsnorm(h, self.norm), *self.head)
