"""Continuous batching on the GPU: the serving engine (mixed prefill + decode
steps, per-bucket decode graphs, preemption under a tight KV pool) gives
every request exactly the greedy tokens it gets when served alone. The W8A8
path is batch-invariant -- per-token quantisation, per-sequence attention,
exact int32 sums -- so this holds bit for bit."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _requests(S, vocab):
    g = torch.Generator().manual_seed(11)
    shapes = [(0, 3, 5), (5, 12, 9), (17, 40, 3), (0, 25, 12), (9, 7, 2), (3, 33, 8), (0, 1, 6)]
    reqs = []
    for i, (pts, t, out) in enumerate(shapes):
        reqs.append(S.Request(rid=i, text_ids=torch.randint(0, vocab, (t,), generator=g).tolist(), max_tokens=out,
                              n_point_rows=pts, point_seed=100 + i))
    return reqs


@pytest.mark.parametrize("num_blocks,max_num_seqs", [(64, 8), (6, 4), (5, 8)])
def test_batched_serving_equals_serving_alone(cuda_device, num_blocks, max_num_seqs):
    from nanopointllm_b200 import runner as R, serving as S, synthetic as Sy
    shape = Sy.TINY
    sd = Sy.llama_weights(shape, seed=0)
    run = R.W8A8LlamaRunner(shape, sd, device=cuda_device, num_blocks=num_blocks, block_size=16)
    reqs = _requests(S, shape.vocab)
    eng = S.ServingEngine(run, max_num_seqs=max_num_seqs, max_num_batched_tokens=96, max_blocks_per_seq=6)
    res = eng.run(reqs)
    assert res["output_tokens"] == sum(q.max_tokens for q in reqs)
    assert all(len(res["outputs"][q.rid]) == q.max_tokens for q in reqs)
    if num_blocks <= 6:
        assert res["preemptions"] > 0  # the tight pool forces recomputation
    assert res["steps"]["decode"] > 0 and res["steps"]["mixed"] > 0
    for q in reqs:
        alone = S.ServingEngine(run, max_blocks_per_seq=6, use_graphs=False).run([q])
        assert alone["outputs"][q.rid] == res["outputs"][q.rid], f"request {q.rid}"
    from nanopointllm_b200 import _lib
    _lib.device_status()


def test_serving_graphs_equal_eager(cuda_device):
    from nanopointllm_b200 import runner as R, serving as S, synthetic as Sy
    shape = Sy.TINY
    sd = Sy.llama_weights(shape, seed=0)
    run = R.W8A8LlamaRunner(shape, sd, device=cuda_device, num_blocks=64, block_size=16)
    reqs = _requests(S, shape.vocab)
    a = S.ServingEngine(run, max_blocks_per_seq=6, use_graphs=True).run(reqs)
    b = S.ServingEngine(run, max_blocks_per_seq=6, use_graphs=False).run(reqs)
    assert a["outputs"] == b["outputs"]
