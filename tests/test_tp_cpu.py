"""Tensor-parallel host logic on CPU: world sizes 2 and 4 over gloo (127.0.0.1).

Each rank slices oracle-quantised full weights with the plan of
nanopointllm_b200.tp (the functions the GPU runner uses), runs its part of a
row-parallel O / down projection and of the column-parallel QKV, gate/up and
LM head with the numpy oracle, and exchanges exactly what the runner
exchanges: the per-token absmax (MAX), the int32 partial accumulators (SUM)
and the LM-head logits (all-gather). The results must equal the unsharded
oracle bit for bit. The GPU runner itself is covered by tests/test_tp_gpu.py.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w8a8 as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, errors) -> None:
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import conftest  # noqa: F401  (registers the package)
        from nanopointllm_b200 import tp
        from nanopointllm_b200.synthetic import LlamaShape

        # world 4 also leaves a rank's intermediate slice ragged (344 = 4 x 86)
        shape = LlamaShape(hidden=256, heads=4, kv_heads=2, head_dim=64, intermediate=336, layers=1, vocab=1001) \
            if world == 2 else LlamaShape(hidden=256, heads=8, kv_heads=4, head_dim=64, intermediate=344, layers=1,
                                          vocab=1001)
        plan = tp.tp_plan(shape, rank, world)
        rng = np.random.default_rng(7)  # same full weights on every rank
        m, hd = 5, shape.head_dim
        w_qkv = rng.standard_normal(((shape.heads + 2 * shape.kv_heads) * hd, shape.hidden)).astype(np.float16)
        w_o = rng.standard_normal((shape.hidden, shape.heads * hd)).astype(np.float16)
        w_g = rng.standard_normal((shape.intermediate, shape.hidden)).astype(np.float16)
        w_d = rng.standard_normal((shape.hidden, shape.intermediate)).astype(np.float16)
        w_v = rng.standard_normal((shape.vocab, shape.hidden)).astype(np.float16)
        x = rng.standard_normal((m, shape.hidden)).astype(np.float16)
        attn = (rng.standard_normal((m, shape.heads * hd)) * 3).astype(np.float16)
        act = (rng.standard_normal((m, shape.intermediate)) * 2).astype(np.float16)
        res = rng.standard_normal((m, shape.hidden)).astype(np.float16)

        def quant(wt):
            q, s = O.per_output_weight_quant(wt)
            return torch.from_numpy(q), torch.from_numpy(s.reshape(-1))

        # column-parallel QKV: this rank's rows of the full result
        qq, qs = quant(w_qkv)
        rows = tp.qkv_rows(shape, plan)
        xq, xs = O.dynamic_per_token_quant(x)
        full, _ = O.w8a8_linear(xq, xs, qq.numpy(), qs.numpy())
        part, _ = O.w8a8_linear(xq, xs, qq[rows].numpy(), qs[rows].numpy())
        np.testing.assert_array_equal(part, full[:, rows.numpy()])

        def row_parallel(x_full, x_local, wq, ws, w_local):
            """x_local / w_local: this rank's columns of the input rows and of
            the full quantised weight wq (per-row scales ws)."""
            # whole-row absmax: MAX over ranks of the local absmax (fp32 bits)
            local = np.abs(x_local.astype(np.float32)).max(axis=1).astype(np.float32).view(np.int32)
            amax = torch.from_numpy(local.copy())
            dist.all_reduce(amax, op=dist.ReduceOp.MAX)
            scale = O.scale_from_absmax(amax.numpy().view(np.float32).reshape(-1, 1))
            fq, fs = O.dynamic_per_token_quant(x_full)
            np.testing.assert_array_equal(scale, fs)
            xq_local = O.quantize_symmetric(x_local, scale)
            acc = torch.from_numpy(O.int_matmul_nt(xq_local, w_local.numpy()).astype(np.int32))
            dist.all_reduce(acc, op=dist.ReduceOp.SUM)  # exact int32 partial sums
            full_acc = O.int_matmul_nt(fq, wq.numpy())
            np.testing.assert_array_equal(acc.numpy(), full_acc)
            out = (O.dequantize(acc.numpy(), scale, ws.numpy()).astype(np.float16).astype(np.float32)
                   + res.astype(np.float32)).astype(np.float16)
            ref, _ = O.w8a8_linear(fq, fs, wq.numpy(), ws.numpy())
            np.testing.assert_array_equal(out, (ref.astype(np.float32) + res.astype(np.float32)).astype(np.float16))

        # row-parallel O over this rank's heads
        oq, os_ = quant(w_o)
        cols = slice(plan.h0 * hd, (plan.h0 + plan.hl) * hd)
        row_parallel(attn, attn[:, cols], oq, os_, oq[:, cols])

        # gate rows / down columns of this rank, zero-padded to a multiple of 64
        gq, gs = quant(w_g)
        sl = slice(plan.i0, plan.i1)
        assert plan.il_pad % 64 == 0 and plan.il_pad >= plan.i1 - plan.i0
        g_local = tp.pad_rows(gq[sl], plan.il_pad)
        assert torch.count_nonzero(g_local[plan.i1 - plan.i0:]) == 0
        dq, ds = quant(w_d)
        d_local = tp.pad_cols(dq[:, sl], plan.il_pad)
        act_local = np.zeros((m, plan.il_pad), np.float16)
        act_local[:, :plan.i1 - plan.i0] = act[:, sl]
        # the padding columns are zero in both operands, so they add nothing
        row_parallel(act, act_local, dq, ds, d_local)

        # vocab-parallel LM head + all-gather
        vq, vs = quant(w_v)
        vrows = slice(plan.v0, plan.v1)
        local_q = tp.pad_rows(vq[vrows], plan.vl_pad)
        local_s = tp.pad_rows(vs[vrows], plan.vl_pad, tp.ZERO_ROW_SCALE)
        logits_local = torch.from_numpy(O.w8a8_linear(xq, xs, local_q.numpy(), local_s.numpy())[0].copy())
        gathered = [torch.empty_like(logits_local) for _ in range(world)]
        dist.all_gather(gathered, logits_local)
        logits = torch.stack(gathered).permute(1, 0, 2).reshape(m, -1)[:, :shape.vocab]
        np.testing.assert_array_equal(logits.numpy(), O.w8a8_linear(xq, xs, vq.numpy(), vs.numpy())[0])
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # reported by the parent
        import traceback
        errors.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")


@pytest.mark.parametrize("world", [2, 4])
def test_tp_sharding_and_exchanges(world):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not msgs, "\n".join(msgs)
    assert all(p.exitcode == 0 for p in procs)


def test_tp_plan_covers_every_row():
    import conftest  # noqa: F401
    from nanopointllm_b200 import tp
    from nanopointllm_b200.synthetic import LLAMA_7B
    for world in (1, 2, 4, 8):
        plans = [tp.tp_plan(LLAMA_7B, r, world) for r in range(world)]
        assert sum(p.hl for p in plans) == LLAMA_7B.heads
        assert [p.i0 for p in plans][1:] == [p.i1 for p in plans][:-1] and plans[-1].i1 == LLAMA_7B.intermediate
        assert all(p.il_pad % 64 == 0 and p.il_pad >= p.i1 - p.i0 for p in plans)
        assert plans[-1].v1 == LLAMA_7B.vocab and all(p.vl_pad * world >= LLAMA_7B.vocab for p in plans)
    with pytest.raises(ValueError):
        tp.tp_plan(LLAMA_7B, 0, 3)  # 32 heads do not split over 3 ranks
