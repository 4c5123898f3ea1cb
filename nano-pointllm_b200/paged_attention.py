"""Paged-KV operators on the GPU, mirroring ``nanopointllm.llama.paged_attention``.

* ``store_kvcache``          - paged_attention.py:353-383 (same signature)
* ``paged_decode_attention`` - paged_attention.py:872-1030 (same signature)
* ``paged_varlen_attention`` - paged_attention.py:1142-1207 (same signature;
                               causal prefill / suffix prefill from the pool)
* ``rope_store_kvcache``     - paged_attention.py:1284-1294 (rotary_fn on q/k of
                               the packed QKV projection, then store_kvcache)

KV pool layout per layer (kv_pool.py:9-24): fp16 [num_blocks, block_size,
Hkv, D]; ``slot_mapping`` int32 (-1 = padding, skipped); ``block_tables`` int32
[B, max_blocks]; ``context_lens`` int32 [B]. CUDA tensors only.
"""
from __future__ import annotations

import torch

from . import _lib as L


def _check_cache(k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    if not (k_cache.is_cuda and v_cache.is_cuda):
        raise ValueError("the paged path runs on CUDA tensors only")
    if k_cache.dtype != torch.float16 or v_cache.dtype != torch.float16:
        raise ValueError("KV caches must be float16")
    if k_cache.shape != v_cache.shape or k_cache.dim() != 4:
        raise ValueError("KV caches must be [num_blocks, block_size, Hkv, D]")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("KV caches must be contiguous")


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """Write key/value [T, Hkv, D] into the pool at ``slot_mapping`` (int32)."""
    _check_cache(k_cache, v_cache)
    t, hkv, d = key.shape
    key = key.reshape(t, hkv * d)
    value = value.reshape(t, hkv * d)
    if key.stride(-1) != 1 or value.stride(-1) != 1 or key.stride(0) != value.stride(0):
        key, value = key.contiguous(), value.contiguous()
    nb, bs = k_cache.shape[:2]
    L.check(L.lib.npl_store_kv(key.data_ptr(), value.data_ptr(), key.stride(0), t, hkv, d,
                               slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), nb, bs,
                               L.stream_ptr(key.device)))


def rope_store_kvcache(qkv: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int,
                       cos_table: torch.Tensor, sin_table: torch.Tensor, positions: torch.Tensor,
                       slot_mapping: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       q_out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed QKV projection output [T, (H + 2*Hkv) * D] -> rotated q [T, H, D];
    rotated k and v stored into the pool. cos/sin: fp16 [max_position, D]."""
    _check_cache(k_cache, v_cache)
    t = qkv.shape[0]
    if q_out is None:
        q_out = torch.empty((t, num_heads, head_dim), dtype=torch.float16, device=qkv.device)
    nb, bs = k_cache.shape[:2]
    L.check(L.lib.npl_rope_store_kv(
        qkv.data_ptr(), qkv.stride(0), t, num_heads, num_kv_heads, head_dim, cos_table.data_ptr(),
        sin_table.data_ptr(), cos_table.shape[0], positions.data_ptr(), slot_mapping.data_ptr(), q_out.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, L.stream_ptr(qkv.device)))
    return q_out


def decode_attention_workspace(device: torch.device, b: int, h: int, d: int, max_blocks: int,
                               block_size: int) -> torch.Tensor:
    nbytes = int(L.lib.npl_decode_attention_workspace_bytes(b, h, d, max_blocks, block_size))
    return L.workspaces.get(device, "decode_attention", nbytes)


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                           num_kv_groups: int, block_n: int | None = None,
                           out: torch.Tensor | None = None, quant_out: tuple | None = None) -> torch.Tensor:
    """Decode-only paged attention (q_len = 1): q fp16 [B, H, D] -> [B, H, D].

    ``block_n`` is accepted for signature compatibility with the reference
    (its Triton tile size); the kernel chooses its own context split.
    ``quant_out = (q8 int8 [B, H*D], scale fp32 [B])`` also receives the
    per-token int8 quantisation of each output row (the O projection input).
    """
    del block_n
    _check_cache(k_cache, v_cache)
    b, h, d = q.shape
    nb, bs, hkv, dk = k_cache.shape
    if dk != d or hkv * num_kv_groups != h:
        raise ValueError("q / KV cache head geometry mismatch")
    if b == 0:
        return q.new_empty((0, h, d))
    q = q.contiguous()
    if out is None:
        out = torch.empty_like(q)
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise ValueError("block_tables and context_lens must be int32")
    max_blocks = block_tables.shape[1]
    ws = decode_attention_workspace(q.device, b, h, d, max_blocks, bs)
    q8, qs = quant_out if quant_out is not None else (None, None)
    L.check(L.lib.npl_paged_decode_attention(
        q.data_ptr(), b, h, hkv, d, k_cache.data_ptr(), v_cache.data_ptr(), nb, bs, block_tables.data_ptr(),
        block_tables.stride(0), max_blocks, context_lens.data_ptr(), float(scale), out.data_ptr(), L.ptr(q8),
        L.ptr(qs), ws.data_ptr(), ws.numel(), L.stream_ptr(q.device)))
    return out


def paged_varlen_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor, q_lens: torch.Tensor,
                           q_offsets: torch.Tensor, scale: float, num_kv_groups: int,
                           block_m: int | None = None, block_n: int | None = None, *,
                           max_q_len: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Varlen paged attention for q_len > 1 prefill / suffix prefill
    (paged_attention.py:1142-1207): q fp16 [total_q, H, D] -> [total_q, H, D].

    ``block_m`` / ``block_n`` are accepted for signature compatibility with the
    reference (its Triton tile sizes); the kernel uses 128 x 128 tiles.
    ``max_q_len`` (>= every q_lens) avoids reading q_lens back to the host.
    """
    del block_m, block_n
    _check_cache(k_cache, v_cache)
    total_q, h, d = q.shape
    nb, bs, hkv, dk = k_cache.shape
    if dk != d or hkv * num_kv_groups != h:
        raise ValueError("q / KV cache head geometry mismatch")
    if total_q == 0:
        return q.new_empty((0, h, d))
    if q.dtype != torch.float16:
        raise ValueError("q must be float16")
    if q.stride(2) != 1 or q.stride(1) != d:
        q = q.contiguous()
    for t in (block_tables, context_lens, q_lens, q_offsets):
        if t.dtype != torch.int32:
            raise ValueError("block_tables, context_lens, q_lens and q_offsets must be int32")
    block_tables = block_tables if block_tables.stride(1) == 1 else block_tables.contiguous()
    context_lens, q_lens, q_offsets = context_lens.contiguous(), q_lens.contiguous(), q_offsets.contiguous()
    if out is None:
        out = torch.empty((total_q, h, d), dtype=torch.float16, device=q.device)
    if max_q_len is None:
        max_q_len = int(q_lens.max().item()) if q_lens.numel() else 0
    L.check(L.lib.npl_paged_prefill_attention(
        q.data_ptr(), q.stride(0), total_q, h, hkv, d, k_cache.data_ptr(), v_cache.data_ptr(), nb, bs,
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], context_lens.data_ptr(),
        q_lens.data_ptr(), q_offsets.data_ptr(), q_lens.numel(), int(max_q_len), float(scale), out.data_ptr(),
        out.stride(0), L.stream_ptr(q.device)))
    return out

