"""Golden vectors for the varlen paged prefill attention, made by the REFERENCE.

Runs the reference's own Triton kernel ``_paged_varlen_attention_kernel``
(nanopointllm/llama/paged_attention.py:1037-1139) in Triton's CPU interpreter
(TRITON_INTERPRET=1; no GPU in the generating container), with the launch
arguments its wrapper ``paged_varlen_attention`` (:1142-1207) computes,
including the default BLOCK_M / BLOCK_N of ``_varlen_blocks`` (:53-63). The
wrapper itself refuses CPU tensors, so the kernel object is launched here.

    NPL_REFERENCE=/path/to/Nano-pointllm python tests/golden/make_prefill_golden.py

Writes tests/golden/prefill_attention.npz: for each case its inputs (q, K/V
pool, block tables, lengths, offsets, scale, kv groups) and the reference's
fp16 output.
"""
from __future__ import annotations

import os
import pathlib
import sys

os.environ["TRITON_INTERPRET"] = "1"  # before triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
REF = os.environ.get("NPL_REFERENCE")  # root of the Nano-pointllm checkout (required)

# (name, H, Hkv, D, block_size, [(q_len, ctx_len), ...], seed)
CASES = [
    ("gqa2_bs16", 4, 2, 128, 16, [(37, 37), (5, 21)], 1),
    ("d64_bs256_suffix", 2, 2, 64, 256, [(200, 300)], 2),
    ("gqa4_multi_tile", 4, 1, 128, 16, [(130, 130), (1, 77), (64, 300)], 3),
]


def run_case(PA, triton, H, Hkv, D, bs, seqs, seed):
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(-(-ctx // bs) for _, ctx in seqs)
    num_blocks = len(seqs) * max_blocks + 3
    k_cache = torch.randn(num_blocks, bs, Hkv, D, generator=g).half()
    v_cache = torch.randn(num_blocks, bs, Hkv, D, generator=g).half()
    perm = torch.randperm(num_blocks, generator=g)
    bt = perm[:len(seqs) * max_blocks].reshape(len(seqs), max_blocks).to(torch.int32)
    q_lens = torch.tensor([ql for ql, _ in seqs], dtype=torch.int32)
    ctx = torch.tensor([c for _, c in seqs], dtype=torch.int32)
    q_off = torch.tensor(np.concatenate([[0], np.cumsum(q_lens.numpy())[:-1]]), dtype=torch.int32)
    total = int(q_lens.sum())
    q = torch.randn(total, H, D, generator=g).half()
    out = torch.empty_like(q)
    scale = D ** -0.5
    block_m, block_n = PA._varlen_blocks(D)
    grid = (triton.cdiv(int(q_lens.max()), block_m), len(seqs), H)
    PA._paged_varlen_attention_kernel[grid](
        q, k_cache, v_cache, bt, ctx, q_lens, q_off, out,
        q.stride(0), q.stride(1), q.stride(2),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), k_cache.stride(3),
        bt.stride(0), bt.stride(1), out.stride(0), out.stride(1), out.stride(2),
        BLOCK_SIZE=bs, HEAD_DIM=D, BLOCK_D=triton.next_power_of_2(D), BLOCK_M=block_m, BLOCK_N=block_n,
        MAX_CONTEXT_LEN=triton.cdiv(int(ctx.max()), block_n) * block_n, NUM_KV_GROUPS=H // Hkv,
        SCALE=float(scale))
    return dict(q=q.numpy(), k_cache=k_cache.numpy(), v_cache=v_cache.numpy(), block_tables=bt.numpy(),
                context_lens=ctx.numpy(), q_lens=q_lens.numpy(), q_offsets=q_off.numpy(),
                scale=np.float32(scale), groups=np.int32(H // Hkv), out=out.numpy())


def main() -> None:
    sys.path.insert(0, str(REF))
    import triton
    from nanopointllm.llama import paged_attention as PA
    arrays = {}
    for name, H, Hkv, D, bs, seqs, seed in CASES:
        for k, v in run_case(PA, triton, H, Hkv, D, bs, seqs, seed).items():
            arrays[f"{name}__{k}"] = v
        print(name, "done")
    np.savez_compressed(HERE / "prefill_attention.npz", cases=np.array([c[0] for c in CASES]), **arrays)


if __name__ == "__main__":
    main()
