"""RoPE cos/sin tables for the rope_store kernel.

The reference feeds ``rotary_fn`` the output of HF ``LlamaRotaryEmbedding``
(transformers 5.5, default rope): fp32 angles ``inv_freq @ position_ids``, then
cos/sin in fp32 rounded to the activation dtype. The tables here are built
once per model with that same op sequence on the host (CPU torch), for every
position up to ``max_position``, and moved to the device; the kernel gathers
rows by position. A decode step then needs no per-step table work.
"""
from __future__ import annotations

import torch


def rope_tables(head_dim: int, max_position: int, theta: float = 10000.0,
                device: torch.device | str = "cpu") -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(max_position, dtype=torch.int64).reshape(1, 1, -1)
    freqs = (inv_freq[None, :, None].float() @ pos.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = (emb.cos() * 1.0).to(torch.float16)[0]
    sin = (emb.sin() * 1.0).to(torch.float16)[0]
    return cos.contiguous().to(device), sin.contiguous().to(device)
