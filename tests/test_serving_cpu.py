"""Serving host logic on CPU (no kernels): KV block accounting, the FIFO
two-queue scheduler with preemption, the data-parallel router and the
metrics gather over gloo (world size 2, 127.0.0.1)."""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _S():
    from nanopointllm_b200 import serving
    return serving


def test_block_manager_accounting():
    S = _S()
    bm = S.BlockManager(num_blocks=6, block_size=4)
    seq = S.Sequence(S.Request(rid=0, text_ids=[1, 2, 3], max_tokens=8, n_point_rows=2))  # 5 positions
    assert bm.blocks_for(seq) == 2 and bm.can_allocate(seq)
    bm.allocate(seq)
    assert len(seq.block_table) == 2 and bm.num_free == 4
    for tok in range(3):  # 6, 7, 8 positions: no new block
        seq.token_ids.append(tok)
        assert bm.can_append(seq)
        bm.may_append(seq)
    assert len(seq.block_table) == 2
    seq.token_ids.append(9)  # 9 positions: the last starts block 3
    bm.may_append(seq)
    assert len(seq.block_table) == 3 and bm.num_free == 3
    bm.deallocate(seq)
    assert bm.num_free == 6 and seq.block_table == []


def _simulate(S, requests, num_blocks, block_size, max_num_seqs, budget):
    """Runs the scheduler with a fake model that samples token = step count."""
    bm = S.BlockManager(num_blocks, block_size)
    sched = S.Scheduler(max_num_seqs, budget, bm)
    seqs = [S.Sequence(q) for q in requests]
    for s in seqs:
        sched.add(s)
    steps = 0
    while not sched.is_finished():
        prefill, decode = sched.schedule()
        assert prefill or decode, "scheduler stalled"
        # every running sequence holds the blocks of all its positions
        for s in prefill + decode:
            assert len(s.block_table) * block_size >= s.num_tokens
        assert len(sched.running) <= max_num_seqs
        sched.postprocess(prefill + decode, [steps] * (len(prefill) + len(decode)), float(steps))
        steps += 1
        assert steps < 10_000
    assert bm.num_free == num_blocks
    return seqs, steps


def test_scheduler_serves_everything_and_preempts_when_blocks_run_out():
    S = _S()
    reqs = [S.Request(rid=i, text_ids=list(range(5 + i)), max_tokens=6 + (i % 3) * 5, n_point_rows=3)
            for i in range(10)]
    # ample pool: no preemption
    seqs, _ = _simulate(S, reqs, num_blocks=200, block_size=4, max_num_seqs=8, budget=64)
    assert all(s.num_completion_tokens == s.req.max_tokens for s in seqs)
    assert sum(s.preemptions for s in seqs) == 0
    # tight pool: sequences are preempted and recomputed, and still finish
    seqs, _ = _simulate(S, reqs, num_blocks=14, block_size=4, max_num_seqs=8, budget=64)
    assert all(s.num_completion_tokens == s.req.max_tokens for s in seqs)
    assert sum(s.preemptions for s in seqs) > 0


def test_scheduler_admission_order_and_budget():
    S = _S()
    bm = S.BlockManager(100, 8)
    sched = S.Scheduler(max_num_seqs=3, max_num_batched_tokens=40, block_manager=bm)
    for i in range(5):
        sched.add(S.Sequence(S.Request(rid=i, text_ids=[0] * 15, max_tokens=2)))
    prefill, decode = sched.schedule()
    assert [s.req.rid for s in prefill] == [0, 1] and decode == []  # 15 + 15 <= 40 < 45
    prefill, decode = sched.schedule()
    assert [s.req.rid for s in prefill] == [2] and [s.req.rid for s in decode] == [0, 1]  # max_num_seqs = 3


def test_route_balances_and_covers():
    S = _S()
    reqs = S.config5_requests(64, vocab=1000, seed=3)
    for world in (1, 2, 3, 8):
        shares = S.route(reqs, world)
        ids = sorted(q.rid for s in shares for q in s)
        assert ids == list(range(64))
        loads = [sum(q.n_point_rows + len(q.text_ids) + q.max_tokens for q in s) for s in shares]
        biggest = max(q.n_point_rows + len(q.text_ids) + q.max_tokens for q in reqs)
        assert max(loads) - min(loads) <= biggest
        assert all(s == sorted(s, key=lambda q: q.rid) for s in shares)
    assert S.route(reqs, 4) == S.route(reqs, 4)  # deterministic


def test_config5_workload_shape():
    S = _S()
    reqs = S.config5_requests(256, vocab=32003)
    assert len(reqs) == 256
    assert all(q.n_point_rows == 513 and 47 <= len(q.text_ids) <= 511 for q in reqs)
    assert {q.max_tokens for q in reqs} == {16, 64, 256}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import conftest  # noqa: F401
        from nanopointllm_b200 import serving as S
        res = {"elapsed_s": 1.0 + rank, "output_tokens": 100 * (rank + 1), "prompt_tokens": 10, "preemptions": rank,
               "ttft_s": {rank * 10 + i: 0.1 * (i + 1) for i in range(4)}}
        out = S.gather_metrics(res)
        if rank == 0:
            assert out["replicas"] == 2 and out["output_tokens"] == 300 and out["elapsed_s"] == 2.0
            assert abs(out["output_tokens_per_s"] - 150.0) < 1e-9
            assert out["preemptions"] == 1 and out["per_replica_elapsed_s"] == [1.0, 2.0]
            assert out["ttft_p50_s"] == pytest.approx(0.3)
        else:
            assert out is None
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        import traceback
        errors.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")


def test_gather_metrics_world2():
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive and not msgs, "\n".join(msgs)


def test_decode_metadata_rows_and_padding():
    """The host metadata of a padded decode step: per sequence its last
    token, position, KV slot and context length, its block table zero-padded;
    padding rows at slot -1 and context 0."""
    S = _S()

    class _Runner:  # what ServingEngine reads from its runner on the host
        num_blocks, block_size, device = 32, 4, "cpu"

    eng = S.ServingEngine(_Runner(), max_num_seqs=4, max_blocks_per_seq=5)
    seqs = []
    for rid, (n_text, n_pts) in enumerate([(3, 2), (9, 0), (1, 6)]):
        s = S.Sequence(S.Request(rid=rid, text_ids=list(range(10 + rid, 10 + rid + n_text)), max_tokens=4,
                                 n_point_rows=n_pts))
        eng.bm.allocate(s)
        s.token_ids.append(100 + rid)  # one generated token: its KV is written by this step
        eng.bm.may_append(s)
        seqs.append(s)
    ids, pos, slots, ctx, bt = eng._decode_metadata(seqs, 8)
    assert ids.tolist() == [100, 101, 102] + [0] * 5
    assert pos.tolist() == [s.num_tokens - 1 for s in seqs] + [0] * 5
    want_slots = [s.block_table[(s.num_tokens - 1) // 4] * 4 + (s.num_tokens - 1) % 4 for s in seqs]
    assert slots.tolist() == want_slots + [-1] * 5
    assert ctx.tolist() == [s.num_tokens for s in seqs] + [0] * 5
    assert bt.shape == (8, 5) and bt.dtype.is_floating_point is False
    for i, s in enumerate(seqs):
        assert bt[i].tolist() == s.block_table + [0] * (5 - len(s.block_table))
    assert bt[3:].abs().sum().item() == 0
    seqs[0].block_table += [1, 2, 3, 4]  # more blocks than a row holds
    with pytest.raises(RuntimeError):
        eng._block_tables(seqs, 4)
