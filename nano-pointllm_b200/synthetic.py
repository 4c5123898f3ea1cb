"""Seeded synthetic inputs for the W8A8 decode path (no datasets, no checkpoints).

The recipes follow the workload descriptions the path is measured on: a single
packed-QKV linear (X ~N(0,1) with 1% outlier channels x20, W ~N(0,0.02)), the
Llama-7B decode MLP block, and a random-init Llama-7B-architecture backbone
(hidden 4096, 32 heads of 128, intermediate 11008, vocab 32003, RoPE theta 1e4)
standing in for the PointLLM-7B LLM, with point embeddings ~N(0,1).

All CPU recipes draw from ``torch.Generator().manual_seed(seed)`` in a fixed
order, so the same tensors are rebuilt on any machine with this torch build;
that is how the golden fixtures avoid storing large inputs.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

import torch


@dataclass(frozen=True)
class LlamaShape:
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    layers: int
    vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-6
    max_position: int = 2048

    def as_dict(self) -> dict:
        return asdict(self)


LLAMA_7B = LlamaShape(hidden=4096, heads=32, kv_heads=32, head_dim=128,
                      intermediate=11008, layers=32, vocab=32003)

# Small model with the 7B head geometry (head_dim 128, no GQA) and a vocab that
# is not a multiple of the 128-row weight tile. Used for model-level parity.
TINY = LlamaShape(hidden=512, heads=4, kv_heads=4, head_dim=128,
                  intermediate=1024, layers=2, vocab=1000, max_position=512)


def config1_inputs(seed: int = 0, m: int = 8, k: int = 4096, n: int = 12288):
    """Single packed-QKV linear: X fp32 [m, k] ~N(0,1) with 1% of channels
    (chosen by randperm) scaled x20; W fp32 [n, k] ~N(0, 0.02)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    idx = torch.randperm(k, generator=g)[: max(1, k // 100)]
    x[:, idx] *= 20.0
    w = torch.randn(n, k, generator=g) * 0.02
    return x, w


def mlp_block_inputs(m: int, seed: int = 1, hidden: int = 4096, inter: int = 11008,
                     device: str = "cpu"):
    """Decode MLP block: x, residual fp16 [m, hidden] ~N(0,1); norm weight
    1+N(0,0.01); gate/up [2*inter, hidden] and down [hidden, inter] ~N(0,0.02)
    (fp16, quantised per output channel by the caller)."""
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(generator=g, device=device)
    x = torch.randn(m, hidden, **kw).half()
    res = torch.randn(m, hidden, **kw).half()
    norm_w = (1.0 + 0.01 * torch.randn(hidden, **kw)).half()
    gate = (torch.randn(inter, hidden, **kw) * 0.02).half()
    up = (torch.randn(inter, hidden, **kw) * 0.02).half()
    down = (torch.randn(hidden, inter, **kw) * 0.02).half()
    return x, res, norm_w, gate, up, down


def llama_weight_names(shape: LlamaShape) -> list[tuple[str, tuple[int, ...], str]]:
    """HF LlamaForCausalLM state-dict names in generation order with (shape, kind)."""
    h, i_, v = shape.hidden, shape.intermediate, shape.vocab
    q_out = shape.heads * shape.head_dim
    kv_out = shape.kv_heads * shape.head_dim
    names = [("model.embed_tokens.weight", (v, h), "linear")]
    for layer in range(shape.layers):
        p = f"model.layers.{layer}."
        names += [
            (p + "input_layernorm.weight", (h,), "norm"),
            (p + "self_attn.q_proj.weight", (q_out, h), "linear"),
            (p + "self_attn.k_proj.weight", (kv_out, h), "linear"),
            (p + "self_attn.v_proj.weight", (kv_out, h), "linear"),
            (p + "self_attn.o_proj.weight", (h, q_out), "linear"),
            (p + "post_attention_layernorm.weight", (h,), "norm"),
            (p + "mlp.gate_proj.weight", (i_, h), "linear"),
            (p + "mlp.up_proj.weight", (i_, h), "linear"),
            (p + "mlp.down_proj.weight", (h, i_), "linear"),
        ]
    names += [("model.norm.weight", (h,), "norm"), ("lm_head.weight", (v, h), "linear")]
    return names


def llama_weights(shape: LlamaShape, seed: int = 0, device: str = "cpu",
                  dtype: torch.dtype = torch.float16) -> dict[str, torch.Tensor]:
    """Random-init weights: linears/embeddings ~N(0, 0.02), norms 1+N(0, 0.1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shp, kind in llama_weight_names(shape):
        t = torch.randn(shp, generator=g, device=device)
        t = 1.0 + 0.1 * t if kind == "norm" else t * 0.02
        out[name] = t.to(dtype)
    return out


def decode_prompts(batch: int, vocab: int, lengths, seed: int = 2) -> list[list[int]]:
    """Token-id prompts, uniform in [0, vocab)."""
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (int(n),), generator=g).tolist() for n in lengths[:batch]]


def permuted_block_tables(batch: int, blocks_per_seq: int, num_blocks: int, seed: int = 3):
    """Disjoint physical blocks per sequence drawn from a random permutation of
    the pool, as int32 [batch, blocks_per_seq]."""
    if batch * blocks_per_seq > num_blocks:
        raise ValueError("KV pool too small for the requested block tables")
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g)[: batch * blocks_per_seq]
    return perm.reshape(batch, blocks_per_seq).to(torch.int32)


class LazyLlamaWeights:
    """Mapping name -> fp16 tensor generated on first access (on ``device``)
    from a per-tensor seed, with the distributions of ``llama_weights``.

    Lets a 7B-shaped random-init model be quantised tensor by tensor without
    ever holding all fp16 weights at once."""

    def __init__(self, shape: LlamaShape, seed: int = 0, device: str = "cuda"):
        self.shape = shape
        self.device = device
        self._meta = {name: (i, shp, kind) for i, (name, shp, kind) in enumerate(llama_weight_names(shape))}
        self.seed = seed

    def __getitem__(self, name: str) -> torch.Tensor:
        i, shp, kind = self._meta[name]
        g = torch.Generator(device=self.device).manual_seed(self.seed * 1_000_003 + i)
        t = torch.randn(shp, generator=g, device=self.device, dtype=torch.float32)
        t = 1.0 + 0.1 * t if kind == "norm" else t * 0.02
        return t.to(torch.float16)

    def __contains__(self, name: str) -> bool:
        return name in self._meta

    def keys(self):
        return self._meta.keys()
