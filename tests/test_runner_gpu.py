"""Model-level parity on the GPU: the W8A8 runner (prefill + decode through
libnpl_w8a8, eager and CUDA graph) against the reference's tiny-Llama
fixtures and the numpy oracle model."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import assert_match_until_tie, golden

pytestmark = pytest.mark.gpu


def _setup(fixture, device):
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    g = golden(fixture)
    shape = S.LlamaShape(**json.loads(str(g["shape"])))
    sd = S.llama_weights(shape, seed=int(g["weight_seed"]))
    prompts = S.decode_prompts(len(g["lengths"]), shape.vocab, g["lengths"].tolist(), seed=int(g["prompt_seed"]))
    run = R.W8A8LlamaRunner(shape, sd, device=device, num_blocks=int(g["num_blocks"]),
                            block_size=int(g["block_size"]))
    return g, shape, prompts, run


def _generate(run, prompts, bt_np, steps, device, graph=False):
    from nanopointllm_b200 import runner as R
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
    R.set_forward_context(R.ForwardContext(slot_mapping=slots, block_tables=bt,
                                           context_lens=torch.tensor(lengths, dtype=torch.int32, device=device),
                                           position_ids=pos, seq_lens=lengths))
    try:
        logits = run.forward(ids, position_ids=pos, last_only=True)[0].float()
    finally:
        R.clear_forward_context()
    dg = None
    if graph:
        dg = R.DecodeGraph(run, len(prompts), bt.shape[1])
    out_tok, out_logits = [], []
    for step in range(steps):
        nxt = logits.argmax(-1)
        out_tok.append(nxt.tolist())
        out_logits.append(logits.cpu().numpy())
        for b in range(len(seqs)):
            seqs[b].append(int(nxt[b]))
        if step == steps - 1:
            break
        ctx = [len(t) for t in seqs]
        ids = torch.tensor([t[-1] for t in seqs], device=device)
        pos = torch.tensor([n - 1 for n in ctx], device=device)
        slots = torch.tensor([slot(b, n - 1) for b, n in enumerate(ctx)], dtype=torch.int32, device=device)
        ctx_t = torch.tensor(ctx, dtype=torch.int32, device=device)
        if dg is not None:
            if dg.graph is None:
                dg.load(ids, pos, slots, ctx_t, bt)
                # capture runs the step twice; restore the slots it wrote twice (same values)
                dg.capture()
            dg.load(ids, pos, slots, ctx_t, bt)
            dg.replay()
            logits = dg.logits[0].float().clone()
        else:
            R.set_forward_context(R.ForwardContext(slot_mapping=slots, block_tables=bt, context_lens=ctx_t,
                                                   position_ids=pos, seq_lens=[1] * len(seqs)))
            try:
                logits = run.forward(ids, position_ids=pos)[0].float()
            finally:
                R.clear_forward_context()
    return np.array(out_tok, np.int32), np.stack(out_logits)


@pytest.mark.parametrize("graph", [False, True])
def test_tiny_model_tokens_match_reference(cuda_device, graph):
    """Against the reference with exact (fp64) prefill attention over prefill
    + 7 decode steps: identical greedy tokens and logits within 5e-2 up to a
    near-tie (reference top-2 closer than 2e-2). The runner's prefill
    attention rounds the probabilities to fp16 for P.V, as the reference's
    CUDA path (its Triton varlen kernel) does: that moves these small
    random-init logits by up to ~0.04 (5e-2 is the bound used against the
    stock reference's own fp16 attention), and a near-tie of the exact model
    may fall either way."""
    g, shape, prompts, run = _setup("tiny_model_fp64_attention.npz", cuda_device)
    steps = g["tokens"].shape[0]
    tokens, logits = _generate(run, prompts, g["block_tables"], steps, cuda_device, graph=graph)
    assert_match_until_tie(tokens, logits, g["tokens"], g["logits"], tie_tol=2e-2, atol=5e-2)
    from nanopointllm_b200 import _lib
    _lib.device_status()


def test_tiny_model_vs_oracle_model(cuda_device):
    """Against the oracle model with the reference's CUDA-path prefill
    attention (oracle.attention, pinned to the reference's Triton kernel):
    same greedy tokens (up to a tie closer than 2e-3) and logits within 3e-2.
    The two prefill attentions agree to one fp16 ulp (128- vs 64-key tiles);
    such a ulp can flip an int8 rounding of the O projection's input, which
    this small random-init model amplifies through RMSNorm (~0.02 seen)."""
    from oracle import model as OM
    g, shape, prompts, run = _setup("tiny_model_fp64_attention.npz", cuda_device)
    from nanopointllm_b200 import synthetic as S
    weights = {k: v.numpy() for k, v in S.llama_weights(shape, seed=int(g["weight_seed"])).items()}
    oracle = OM.W8A8LlamaOracle(weights, shape, int(g["num_blocks"]), int(g["block_size"]), prefill="varlen")
    ot, ol = OM.greedy_generate(oracle, prompts, g["block_tables"], steps=4)
    tokens, logits = _generate(run, prompts, g["block_tables"], 4, cuda_device)
    assert_match_until_tie(tokens, logits, ot, ol, tie_tol=2e-3, atol=3e-2, min_steps=4)


def test_graph_replay_equals_eager(cuda_device):
    g, shape, prompts, run = _setup("tiny_model.npz", cuda_device)
    t_e, l_e = _generate(run, prompts, g["block_tables"], 5, cuda_device, graph=False)
    g, shape, prompts, run = _setup("tiny_model.npz", cuda_device)
    t_g, l_g = _generate(run, prompts, g["block_tables"], 5, cuda_device, graph=True)
    np.testing.assert_array_equal(t_e, t_g)
    np.testing.assert_array_equal(l_e, l_g)
