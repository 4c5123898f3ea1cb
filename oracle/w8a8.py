"""numpy restatement of the reference W8A8 contract and the decode-layer math.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker for the CUDA
kernels, never the product path.

Each function cites the reference code it restates (paths relative to the
nanopointllm project root). Where the reference leaves an order of floating
point operations to its library (torch's fp32 sum inside ``mean``; torch's
CPU ``exp``), the oracle fixes one exact definition and says so; the CUDA
kernels implement the same definition, so kernel == oracle bit for bit, and
the oracle is pinned to the reference by the golden fixtures with a stated
mismatch bound.
"""
from __future__ import annotations

import numpy as np

# w8a8.py:14-30 (W8A8Contract): symmetric [-127, 127], round-to-nearest-even,
# fp16-stored scales, signed int32 accumulator, bias added after dequant in fp.
QMIN = -127
QMAX = 127
FP16_TINY = np.float32(np.finfo(np.float16).tiny)  # 2**-14
F32 = np.float32
F16 = np.float16


def quantize_symmetric(values, scale) -> np.ndarray:
    """w8a8.py:33-43: int8(clamp(round(v.float() / s.float()), -127, 127)).

    ``round`` is ties-to-even (torch.round == np.rint); the division is one
    IEEE fp32 division.
    """
    s = np.asarray(scale, dtype=F32)
    if np.any(s <= 0):
        raise ValueError("quantization scale must be positive")
    v = np.asarray(values).astype(F32)
    q = np.rint(v / s)
    return np.clip(q, QMIN, QMAX).astype(np.int8)


def scale_from_absmax(absmax) -> np.ndarray:
    """w8a8.py:46-50: max(absmax, fp16.tiny) / 127 -> fp16 -> fp32, >= fp16.tiny."""
    raw = np.maximum(np.asarray(absmax).astype(F32), FP16_TINY) / F32(QMAX)
    return np.maximum(raw.astype(F16).astype(F32), FP16_TINY)


def per_output_weight_quant(weight) -> tuple[np.ndarray, np.ndarray]:
    """w8a8.py:53-62 (per_output_weight_qdq): per-row scale and int8 rows.

    Returns (qweight int8 [N, K], scales fp32 [N]); the dequantised weight the
    reference also returns is ``qweight * scales[:, None]``.
    """
    w = np.asarray(weight).astype(F32)
    rows = w.reshape(w.shape[0], -1)
    scales = scale_from_absmax(np.abs(rows).max(axis=1))
    q = quantize_symmetric(rows, scales[:, None])
    return q.reshape(w.shape), scales


def dynamic_per_token_quant(values) -> tuple[np.ndarray, np.ndarray]:
    """w8a8.py:106-115 (dynamic_per_token_activation_qdq), quantise step.

    Returns (q int8 [..., K], scales fp32 [..., 1]).
    """
    v = np.asarray(values)
    scales = scale_from_absmax(np.abs(v.astype(F32)).max(axis=-1, keepdims=True))
    return quantize_symmetric(v, scales), scales


def int_matmul_nt(qa: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """w8a8.py:130-132: int32(qa) @ int32(qw).T.

    Evaluated with torch's CPU float32 matmul (the reference computes on torch
    CPU too) over slices of 1024 columns, which is exact: every product is an
    integer of magnitude <= 127**2 and every partial sum of a slice one of
    magnitude <= 1024 * 127**2 < 2**24, so no fp32 rounding occurs in any
    summation order; the slices are then added in int64.
    """
    import torch

    k = qa.shape[-1]
    if k * QMAX * QMAX >= 1 << 31:  # w8a8.py:152-153
        raise OverflowError("worst-case dot product exceeds signed INT32")
    a32 = torch.from_numpy(np.ascontiguousarray(qa.reshape(-1, k))).float()
    w32 = torch.from_numpy(np.ascontiguousarray(qw)).float()
    acc = torch.zeros((a32.shape[0], w32.shape[0]), dtype=torch.int64)
    for k0 in range(0, k, 1024):
        acc += (a32[:, k0:k0 + 1024] @ w32[:, k0:k0 + 1024].T).long()
    return acc.int().numpy()


def dequantize(acc, act_scale, w_scale, bias=None) -> np.ndarray:
    """w8a8.py:133-137: ((float)acc * s_a) * s_w (+ bias), three fp32 roundings."""
    out = np.asarray(acc).astype(F32)
    out = out * np.asarray(act_scale, F32).reshape(-1, 1)
    out = out * np.asarray(w_scale, F32).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, F32).reshape(1, -1)
    return out


def integer_linear_per_output_reference(values, weight, *, activation_scale, bias=None):
    """w8a8.py:118-139: returns (out fp32, acc int32) like the reference golden."""
    values = np.asarray(values)
    weight = np.asarray(weight)
    if values.shape[-1] != weight.shape[1] or weight.ndim != 2:
        raise ValueError("linear input/weight shapes do not match")
    qa = quantize_symmetric(values, activation_scale)
    qw, ws = per_output_weight_quant(weight)
    acc = int_matmul_nt(qa, qw)
    sa = np.asarray(activation_scale, F32)
    sa = np.full((acc.shape[0],), sa.reshape(()), F32) if sa.size == 1 else sa.reshape(-1)
    out = dequantize(acc, sa, ws, bias)
    lead = values.shape[:-1]
    return out.reshape(*lead, weight.shape[0]), acc.reshape(*lead, weight.shape[0])


def w8a8_linear(qa, sa, qw, sw, bias=None, out_dtype=F16) -> tuple[np.ndarray, np.ndarray]:
    """The decode linear on pre-quantised operands: (out, acc).

    ``out`` is the fp32 dequantised value rounded once to ``out_dtype`` (the
    fp16 module output of the eager reference path).
    """
    acc = int_matmul_nt(qa, qw)
    out = dequantize(acc, np.asarray(sa, F32).reshape(-1), sw, bias)
    return out.astype(out_dtype), acc


# --------------------------------------------------------------------------
# fp16 layer math of the eager lightweight runner
# --------------------------------------------------------------------------

def rms_inv(x16: np.ndarray, eps: float) -> np.ndarray:
    """1 / sqrt(mean(x^2) + eps) in fp32, per row.

    Reference: lightweight_runner.py:242-245, ``x.pow(2).mean(-1) + eps`` then
    ``torch.rsqrt`` (an IEEE 1/sqrt on CPU). Torch's fp32 sum order inside
    ``mean`` is a library detail; the oracle defines the mean as the fp64 sum of
    the (exact) fp32 squares divided by K, rounded once to fp32.
    """
    xf = x16.astype(F32).astype(np.float64)
    mean = (xf * xf).sum(axis=-1, keepdims=True) / x16.shape[-1]
    v = mean.astype(F32) + F32(eps)
    return F32(1.0) / np.sqrt(v.astype(F32))


def rmsnorm(x16: np.ndarray, w16: np.ndarray, eps: float) -> np.ndarray:
    """lightweight_runner.py:239-245 (LightweightRMSNorm.forward, eager):
    fp32 normalise -> round to fp16 -> fp16 weight * x (one fp16 rounding)."""
    y = (x16.astype(F32) * rms_inv(x16, eps)).astype(F16)
    return (w16.astype(F32) * y.astype(F32)).astype(F16)


def rmsnorm_quant(x16, w16, eps, residual16=None):
    """RMSNorm (optionally of x + residual, lightweight_runner.py:259-260, fp16
    add) followed by per-token quantisation (w8a8.py:106-115).

    Returns (q int8, scale fp32 [M], normed fp16, summed fp16 or None).
    """
    summed = None
    if residual16 is not None:
        summed = (x16.astype(F32) + residual16.astype(F32)).astype(F16)
        x16 = summed
    normed = rmsnorm(x16, w16, eps)
    q, s = dynamic_per_token_quant(normed)
    return q, s.reshape(-1), normed, summed


def silu_f16(g16: np.ndarray) -> np.ndarray:
    """SiLU of fp16 values, rounded once to fp16.

    Reference: ``act_fn(gate)`` = torch SiLU on fp16 (lightweight_runner.py:358,
    396), which evaluates g / (1 + exp(-g)) in fp32 with the CPU library exp.
    The oracle evaluates the same formula in fp64 and rounds directly to fp16.
    """
    g = g16.astype(np.float64)
    return (g / (1.0 + np.exp(-g))).astype(F16)


def silu_mul(g16: np.ndarray, u16: np.ndarray) -> np.ndarray:
    """lightweight_runner.py:358 ``act_fn(gate) * up`` in fp16."""
    return (silu_f16(g16).astype(F32) * u16.astype(F32)).astype(F16)


def rotate_half(x):
    half = x.shape[-1] // 2
    return np.concatenate([-x[..., half:], x[..., :half]], axis=-1)


def apply_rope(x16: np.ndarray, cos16: np.ndarray, sin16: np.ndarray) -> np.ndarray:
    """HF ``apply_rotary_pos_emb`` (called through ``rotary_fn``,
    paged_attention.py:1286-1292) on fp16 tensors: q*cos + rotate_half(q)*sin,
    each op rounded to fp16. x [T, H, D], cos/sin [T, D]."""
    c = cos16[:, None, :].astype(F32)
    s = sin16[:, None, :].astype(F32)
    a = (x16.astype(F32) * c).astype(F16)
    b = (rotate_half(x16).astype(F32) * s).astype(F16)
    return (a.astype(F32) + b.astype(F32)).astype(F16)


def rope_tables(positions, head_dim: int, theta: float = 10000.0):
    """HF LlamaRotaryEmbedding.forward (default rope, transformers 5.5): fp32
    angles ``inv_freq @ positions`` (a k=1 matmul), ``cat(freqs, freqs)``,
    cos/sin in fp32, rounded to fp16. Returns (cos16, sin16) [T, D].

    Evaluated with the same torch CPU ops as the reference so the tables are
    bit-identical to the ones the reference feeds ``rotary_fn``.
    """
    import torch

    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.int64).reshape(1, 1, -1)
    freqs = (inv_freq[None, :, None].float() @ pos.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = (emb.cos() * 1.0).to(torch.float16)[0].numpy()
    sin = (emb.sin() * 1.0).to(torch.float16)[0].numpy()
    return cos, sin


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """paged_attention.py:386-401 (_store_kvcache_pytorch): write token t to
    slot_mapping[t] (block = slot // block_size, offset = slot % block_size);
    negative slots are padding and are skipped."""
    block_size = k_cache.shape[1]
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot < 0:
            continue
        k_cache[slot // block_size, slot % block_size] = key[t]
        v_cache[slot // block_size, slot % block_size] = value[t]


def paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale, num_kv_groups=1,
                           dtype=np.float64):
    """paged_attention.py:846-869 (_paged_decode_attention_pytorch), evaluated
    in ``dtype``: float64 (the exact reference point), or float32, the
    arithmetic type the reference's SDPA and Triton decode kernels use.

    q [B, H, D]; caches [num_blocks, block_size, Hkv, D]; returns [B, H, D]
    in ``dtype``. A row with context_len 0 (a padded bucket row) returns zeros.
    """
    B, H, D = q.shape
    block_size = k_cache.shape[1]
    out = np.zeros((B, H, D), dtype=dtype)
    for b in range(B):
        n = int(context_lens[b])
        if n <= 0:
            continue
        nblk = (n + block_size - 1) // block_size
        bt = np.asarray(block_tables[b, :nblk])
        k = k_cache[bt].reshape(-1, k_cache.shape[2], D)[:n].astype(dtype)
        v = v_cache[bt].reshape(-1, v_cache.shape[2], D)[:n].astype(dtype)
        for h in range(H):
            kh = h // num_kv_groups
            s = k[:, kh, :] @ q[b, h].astype(dtype) * dtype(scale)
            p = np.exp(s - s.max())
            out[b, h] = (p[:, None] * v[:, kh, :]).sum(0) / p.sum()
    return out
