"""numpy restatement of the reference's varlen paged prefill attention.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for
npl_paged_prefill_attention, never the product path.

Restates ``_paged_varlen_attention_kernel`` (nanopointllm/llama/
paged_attention.py:1037-1139), as launched by ``paged_varlen_attention``
(:1142-1207) with its default key tile BLOCK_N = 64 (``_varlen_blocks``,
:53-63). Per sequence b, head h (kv head h // groups), query row j at absolute
position ctx - q_len + j:

  for each 64-key tile (keys past the context read as zero, :1093-1104):
    s     = fp32(q . k) * scale, masked to -FLT_MAX unless key < ctx and
            key <= the query's position                        (:1106-1108)
    m'    = max(m, rowmax(s));  p = exp(s - m');  alpha = exp(m - m')
    acc   = acc * alpha + fp32(fp16(p) . v)                    (:1110-1113)
    l     = l * alpha + sum(p)
  out = fp16(acc / l)                                          (:1116-1124)

The dot products run in float64 here (the reference's are fp32 sums of exact
fp16 products; the kernel under test sums in a different order, so no fp32
order is more "right" than another); everything else is fp32 as above.
"""
from __future__ import annotations

import numpy as np

F16 = np.float16
F32 = np.float32
F64 = np.float64
NEG = F32(-3.4028234663852886e38)


def paged_varlen_attention(q, k_cache, v_cache, block_tables, context_lens, q_lens, q_offsets, scale: float,
                           num_kv_groups: int, block_n: int = 64) -> np.ndarray:
    """q [total_q, H, D] fp16; caches [num_blocks, block_size, Hkv, D] fp16;
    returns fp16 [total_q, H, D] (rows of no sequence stay zero)."""
    q = np.asarray(q, F16)
    total_q, H, D = q.shape
    bs = k_cache.shape[1]
    out = np.zeros((total_q, H, D), F16)
    scale = F32(scale)
    head_kv = np.arange(H) // num_kv_groups
    for b in range(len(q_lens)):
        q_len, ctx, off = int(q_lens[b]), int(context_lens[b]), int(q_offsets[b])
        if q_len <= 0:
            continue
        prefix = ctx - q_len
        n_pad = -(-max(ctx, 1) // block_n) * block_n
        keys = np.arange(n_pad)
        blk = np.where(keys < ctx, np.asarray(block_tables[b])[np.minimum(keys // bs, len(block_tables[b]) - 1)], 0)
        valid = keys < ctx
        k_all = np.where(valid[:, None, None], k_cache[blk, keys % bs], 0).astype(F16)  # [n_pad, Hkv, D]
        v_all = np.where(valid[:, None, None], v_cache[blk, keys % bs], 0).astype(F16)
        q_pos = prefix + np.arange(q_len)
        # every head at once: [H, q_len, D] queries, [H, n_pad, D] keys/values
        qh = q[off:off + q_len].astype(F64).transpose(1, 0, 2)
        kh_all = k_all[:, head_kv].astype(F64).transpose(1, 0, 2)
        vh_all = v_all[:, head_kv].astype(F64).transpose(1, 0, 2)
        m = np.full((H, q_len), NEG, F32)
        l = np.zeros((H, q_len), F32)
        acc = np.zeros((H, q_len, D), F32)
        for start in range(0, n_pad, block_n):
            if start > q_pos[-1]:
                break  # every key of this and later tiles is masked for every query: p = 0, alpha = 1
            kt = kh_all[:, start:start + block_n]
            vt = vh_all[:, start:start + block_n]
            pos = start + np.arange(block_n)
            s = (qh @ kt.transpose(0, 2, 1)).astype(F32) * scale
            allowed = (pos[None, :] < ctx) & (pos[None, :] <= q_pos[:, None])
            s = np.where(allowed[None], s, NEG)
            m_new = np.maximum(m, s.max(axis=-1))
            p = np.exp(s - m_new[..., None], dtype=F32)
            alpha = np.exp(m - m_new, dtype=F32)
            pv = (p.astype(F16).astype(F64) @ vt).astype(F32)
            acc = acc * alpha[..., None] + pv
            l = l * alpha + p.sum(axis=-1, dtype=F32)
            m = m_new
        out[off:off + q_len] = (acc / l[..., None]).astype(F16).transpose(1, 0, 2)
    return out
