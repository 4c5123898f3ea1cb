"""The runner built the way the reference engine would build it: from an HF
LlamaForCausalLM and a KV-pool tensor in the reference's layout
([2, layers, num_blocks, block_size, Hkv, D], kv_pool.py:9-24), reading the
per-step metadata from a ForwardContext object of the reference's own class
shape (forward_context.py:10-24, including its nano-vllm fields) through a
context getter the engine passes in."""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


@dataclass
class EngineForwardContext:
    """The field list of nanopointllm/engine/forward_context.py:10-24."""
    slot_mapping: torch.Tensor
    block_tables: Optional[torch.Tensor]
    context_lens: Optional[torch.Tensor]
    position_ids: Optional[torch.Tensor] = None
    seq_lens: list = field(default_factory=list)
    num_prefill_tokens: int = 0
    num_prefill_seqs: int = 0
    cu_seqlens_q: Optional[torch.Tensor] = None
    cu_seqlens_k: Optional[torch.Tensor] = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0


_engine_ctx = threading.local()


def engine_get_forward_context():
    return getattr(_engine_ctx, "value", None)


def _hf_model(shape, sd, device):
    import transformers
    cfg = transformers.LlamaConfig(
        hidden_size=shape.hidden, intermediate_size=shape.intermediate, num_hidden_layers=shape.layers,
        num_attention_heads=shape.heads, num_key_value_heads=shape.kv_heads, head_dim=shape.head_dim,
        vocab_size=shape.vocab, max_position_embeddings=shape.max_position, rms_norm_eps=shape.eps,
        tie_word_embeddings=False, rope_theta=shape.rope_theta)
    with torch.device(device):
        model = transformers.LlamaForCausalLM(cfg).to(torch.float16)
    model.load_state_dict({k: v.to(device) for k, v in sd.items()})
    return model


def _steps(run, prompts, bt_np, steps, device, set_ctx, clear_ctx, make_ctx):
    """Prefill + greedy decode, the metadata passed through set_ctx(make_ctx(...))."""
    bs = run.block_size
    bt = torch.from_numpy(bt_np).to(device)

    def slot(b, p):
        return int(bt_np[b, p // bs]) * bs + p % bs

    lengths = [len(p) for p in prompts]
    seqs = [list(p) for p in prompts]
    ids = torch.tensor([t for p in prompts for t in p], device=device)
    pos = torch.cat([torch.arange(n) for n in lengths]).to(device)
    slots = torch.tensor([slot(b, p) for b, n in enumerate(lengths) for p in range(n)], dtype=torch.int32,
                         device=device)
    ctx_lens = torch.tensor(lengths, dtype=torch.int32, device=device)
    out = []
    for step in range(steps):
        set_ctx(make_ctx(slots, bt, ctx_lens, pos.reshape(1, -1), lengths))
        try:
            logits = run.forward(ids, position_ids=pos, last_only=step == 0)[0].float()
        finally:
            clear_ctx()
        out.append(logits.cpu().numpy())
        nxt = logits.argmax(-1).tolist()
        for b in range(len(seqs)):
            seqs[b].append(int(nxt[b]))
        lengths = [1] * len(seqs)
        ctx = [len(t) for t in seqs]
        ids = torch.tensor([t[-1] for t in seqs], device=device)
        pos = torch.tensor([n - 1 for n in ctx], device=device)
        slots = torch.tensor([slot(b, n - 1) for b, n in enumerate(ctx)], dtype=torch.int32, device=device)
        ctx_lens = torch.tensor(ctx, dtype=torch.int32, device=device)
    return np.stack(out)


def test_from_hf_with_engine_context_equals_state_dict_runner(cuda_device):
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    g = golden("tiny_model.npz")
    shape = S.TINY
    sd = S.llama_weights(shape, seed=int(g["weight_seed"]))
    prompts = S.decode_prompts(len(g["lengths"]), shape.vocab, g["lengths"].tolist(), seed=int(g["prompt_seed"]))
    nb, bs = int(g["num_blocks"]), int(g["block_size"])

    # the engine's objects: HF model, KV pool tensor, its own context class and getter
    model = _hf_model(shape, sd, cuda_device)
    pool = torch.zeros(2, shape.layers, nb, bs, shape.kv_heads, shape.head_dim, dtype=torch.float16,
                       device=cuda_device)
    run = R.W8A8LlamaRunner.from_hf(model, pool, forward_context=engine_get_forward_context)
    assert run.shape == shape and run.kv_pool.data_ptr() == pool.data_ptr()

    def set_engine(ctx):
        _engine_ctx.value = ctx

    def clear_engine():
        _engine_ctx.value = None

    def engine_ctx(slots, bt, ctx_lens, pos, lens):
        return EngineForwardContext(slot_mapping=slots, block_tables=bt, context_lens=ctx_lens,
                                    position_ids=pos, seq_lens=list(lens),
                                    num_prefill_seqs=sum(n > 1 for n in lens))

    got = _steps(run, prompts, g["block_tables"], 4, cuda_device, set_engine, clear_engine, engine_ctx)

    ref_run = R.W8A8LlamaRunner(shape, sd, device=cuda_device, num_blocks=nb, block_size=bs)

    def own_ctx(slots, bt, ctx_lens, pos, lens):
        return R.ForwardContext(slot_mapping=slots, block_tables=bt, context_lens=ctx_lens, position_ids=pos,
                                seq_lens=list(lens))

    want = _steps(ref_run, prompts, g["block_tables"], 4, cuda_device, R.set_forward_context,
                  R.clear_forward_context, own_ctx)
    np.testing.assert_array_equal(got, want)
    # the engine's getter is the one read: nothing was set in the runner module's own slot
    assert R.get_forward_context() is None
