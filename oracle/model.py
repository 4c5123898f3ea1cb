"""numpy W8A8 Llama forward over a paged KV pool (prefill + decode).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the eager reference path that the W8A8 golden is defined on:
``LightweightLlamaRunner.forward`` (lightweight_runner.py:625-736) with
``LightweightLlamaLayer.forward`` (:480-560, eager branch), ``PagedLlamaAttention``
(paged_attention.py:1271-1488: q/k/v projections, rotary_fn, store_kvcache,
per-sequence attention over the pool -- float64 as on its CPU path, or its
CUDA path's varlen prefill kernel, oracle.attention -- o_proj), the
non-packed MLP
(lightweight_runner.py:389-404), the final norm and the LM head, where every
Linear is the integer golden of w8a8.py:118-139 on per-token dynamic int8
activations and per-output-channel int8 weights.
"""
from __future__ import annotations

import numpy as np

from . import attention as OA
from . import w8a8 as O

F16 = np.float16
F32 = np.float32


class W8A8LlamaOracle:
    def __init__(self, weights: dict, shape, k_cache_blocks: int, block_size: int, prefill: str = "exact",
                 varlen_block_n: int = 64, quantized: dict | None = None,
                 decode_dtype=np.float64):
        """prefill: "exact" evaluates multi-token rows in float64 (the
        reference's CPU path, SDPA per sequence); "varlen" restates its CUDA
        path, the Triton varlen kernel (oracle.attention), with key tiles of
        ``varlen_block_n`` (the kernel's BLOCK_N: 64 by default for head_dim
        128, NANOPOINTLLM_VARLEN_BLOCK_N selects another, paged_attention.py:53-63).

        ``quantized``: name -> (int8 [N, K], fp32 scales [N]) of Linears
        already quantised per output channel (checked elsewhere against
        per_output_weight_quant); ``weights`` then needs only the embedding
        and the norms. ``decode_dtype``: arithmetic of single-token rows'
        attention (float64, or the reference kernels' float32)."""
        if prefill not in ("exact", "varlen"):
            raise ValueError("prefill must be 'exact' or 'varlen'")
        self.prefill = prefill
        self.varlen_block_n = varlen_block_n
        self.decode_dtype = decode_dtype
        self.s = shape
        self.w = {k: np.asarray(v) for k, v in weights.items()}
        self.q = dict(quantized or {})
        for name, arr in self.w.items():
            if arr.ndim == 2 and name != "model.embed_tokens.weight" and name not in self.q:
                self.q[name] = O.per_output_weight_quant(arr)
        self.block_size = block_size
        kv_shape = (shape.layers, k_cache_blocks, block_size, shape.kv_heads, shape.head_dim)
        self.k_cache = np.zeros(kv_shape, F16)
        self.v_cache = np.zeros(kv_shape, F16)
        pos = np.arange(shape.max_position)
        self.cos, self.sin = O.rope_tables(pos, shape.head_dim, shape.rope_theta)

    def linear(self, name: str, x16: np.ndarray) -> np.ndarray:
        qa, sa = O.dynamic_per_token_quant(x16)
        qw, sw = self.q[name]
        out, _ = O.w8a8_linear(qa, sa, qw, sw)
        return out

    def attention(self, layer, q, seq_lens, context_lens, block_tables):
        """Per-sequence attention over the pool, causal for multi-token rows
        (paged_attention.py:1443-1487), decode form for single-token rows."""
        s = self.s
        groups = s.heads // s.kv_heads
        scale = s.head_dim ** -0.5
        out = np.zeros((q.shape[0], s.heads, s.head_dim), np.float64)
        off = 0
        kc, vc = self.k_cache[layer], self.v_cache[layer]
        starts = np.concatenate([[0], np.cumsum(seq_lens)[:-1]]).astype(np.int32)
        if self.prefill == "varlen":  # paged_attention.py:1406-1433
            pre = [b for b, n in enumerate(seq_lens) if n > 1]
            if pre:
                va = OA.paged_varlen_attention(
                    q, kc, vc, np.asarray(block_tables)[pre], np.asarray(context_lens, np.int32)[pre],
                    np.asarray(seq_lens, np.int32)[pre], starts[pre], scale, groups, block_n=self.varlen_block_n)
                for b in pre:
                    out[starts[b]:starts[b] + seq_lens[b]] = va[starts[b]:starts[b] + seq_lens[b]]
        for b, qlen in enumerate(seq_lens):
            if self.prefill == "varlen" and qlen > 1:
                off += qlen
                continue
            n = int(context_lens[b])
            nblk = (n + self.block_size - 1) // self.block_size
            bt = block_tables[b, :nblk]
            dt = self.decode_dtype if qlen == 1 else np.float64
            k = kc[bt].reshape(-1, s.kv_heads, s.head_dim)[:n].astype(dt)
            v = vc[bt].reshape(-1, s.kv_heads, s.head_dim)[:n].astype(dt)
            prefix = n - qlen
            for j in range(qlen):
                visible = prefix + j + 1
                for h in range(s.heads):
                    kh = h // groups
                    sc = k[:visible, kh] @ q[off + j, h].astype(dt) * dt(scale)
                    p = np.exp(sc - sc.max())
                    out[off + j, h] = (p[:, None] * v[:visible, kh]).sum(0) / p.sum()
            off += qlen
        return out.astype(F16)

    def forward(self, ids, positions, slot_mapping, seq_lens, context_lens, block_tables, *, embeds=None,
                rows=None):
        """Returns fp16 logits [T, vocab] for the flattened new tokens (only
        for the token indices ``rows`` when given, as the runner's
        ``last_only``). ``embeds`` [T, hidden] fp16 replaces the embedding
        lookup of ``ids`` (the engine's inputs_embeds with point rows,
        lightweight_runner.py:625-650)."""
        s = self.s
        h = np.asarray(embeds, F16) if embeds is not None else self.w["model.embed_tokens.weight"][np.asarray(ids)]
        cos, sin = self.cos[positions], self.sin[positions]
        T = h.shape[0]
        for layer in range(s.layers):
            p = f"model.layers.{layer}."
            x = O.rmsnorm(h, self.w[p + "input_layernorm.weight"], s.eps)
            q = self.linear(p + "self_attn.q_proj.weight", x).reshape(T, s.heads, s.head_dim)
            k = self.linear(p + "self_attn.k_proj.weight", x).reshape(T, s.kv_heads, s.head_dim)
            v = self.linear(p + "self_attn.v_proj.weight", x).reshape(T, s.kv_heads, s.head_dim)
            q = O.apply_rope(q, cos, sin)
            k = O.apply_rope(k, cos, sin)
            O.store_kvcache(k, v, self.k_cache[layer], self.v_cache[layer], slot_mapping)
            a = self.attention(layer, q, seq_lens, context_lens, block_tables).reshape(T, -1)
            o = self.linear(p + "self_attn.o_proj.weight", a)
            h = (h.astype(F32) + o.astype(F32)).astype(F16)
            x = O.rmsnorm(h, self.w[p + "post_attention_layernorm.weight"], s.eps)
            g = self.linear(p + "mlp.gate_proj.weight", x)
            u = self.linear(p + "mlp.up_proj.weight", x)
            d = self.linear(p + "mlp.down_proj.weight", O.silu_mul(g, u))
            h = (h.astype(F32) + d.astype(F32)).astype(F16)
        if rows is not None:
            h = h[np.asarray(rows)]
        x = O.rmsnorm(h, self.w["model.norm.weight"], s.eps)
        return self.linear("lm_head.weight", x)


def greedy_generate(oracle: W8A8LlamaOracle, prompts, block_tables, steps: int, embeds=None):
    """Prefill all prompts in one flattened pass (``embeds`` [T, hidden]
    replacing their embedding rows when given), then ``steps - 1`` batched
    decode steps; returns (tokens [steps, B], logits [steps, B, V] fp32)."""
    bs = oracle.block_size
    bt = np.asarray(block_tables)

    def slot(b, p):
        return int(bt[b, p // bs]) * bs + p % bs

    lengths = [len(p) for p in prompts]
    seqs = [list(p) for p in prompts]
    ids = [t for p in prompts for t in p]
    pos = np.concatenate([np.arange(n) for n in lengths])
    slots = np.array([slot(b, p) for b, n in enumerate(lengths) for p in range(n)])
    last = np.cumsum(lengths) - 1
    lg = oracle.forward(ids, pos, slots, lengths, lengths, bt, embeds=embeds, rows=last).astype(F32)
    out_tok, out_logits = [], []
    for _ in range(steps):
        nxt = lg.argmax(-1)
        out_tok.append(nxt.tolist())
        out_logits.append(lg)
        for b in range(len(seqs)):
            seqs[b].append(int(nxt[b]))
        if len(out_tok) == steps:
            break
        ctx = [len(t) for t in seqs]
        ids = [t[-1] for t in seqs]
        pos = np.array([n - 1 for n in ctx])
        slots = np.array([slot(b, n - 1) for b, n in enumerate(ctx)])
        lg = oracle.forward(ids, pos, slots, [1] * len(seqs), ctx, bt).astype(F32)
    return np.array(out_tok, np.int32), np.stack(out_logits)
