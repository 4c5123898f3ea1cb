"""Tensor-parallel runner on 2 GPUs (NCCL, one process per GPU): prefill and
greedy decode of the tiny Llama, eager and CUDA graph, bit-identical to the
single-GPU W8A8LlamaRunner on the same weights, built from the float weights
and from a checksummed int8 package (skipped with fewer than two GPUs)."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, pkg_dir: str, errors) -> None:
    import torch.distributed as dist
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        import conftest  # noqa: F401  (registers the package)
        from test_runner_gpu import _generate
        from nanopointllm_b200 import runner as R, synthetic as S, tp as TP, _lib
        shape = S.TINY
        sd = S.llama_weights(shape, seed=0)
        lengths = [37, 5, 64, 19]
        prompts = S.decode_prompts(len(lengths), shape.vocab, lengths, seed=2)
        bs, per_seq = 16, 6
        bt = S.permuted_block_tables(len(lengths), per_seq, len(lengths) * per_seq, seed=3).numpy()
        full = R.W8A8LlamaRunner(shape, sd, device=dev, num_blocks=len(lengths) * per_seq, block_size=bs)
        t_ref, l_ref = _generate(full, prompts, bt, 5, dev)
        # decode steps through the NVLink peer-memory exchanges (eager and
        # graph), and through the NCCL all-reduces
        for graph, peer in ((False, True), (True, True), (True, False)):
            run = TP.W8A8TPLlamaRunner(shape, sd, device=dev, num_blocks=len(lengths) * per_seq, block_size=bs,
                                       peer_exchange=peer)
            assert (run.xchg is not None) == peer
            t_tp, l_tp = _generate(run, prompts, bt, 5, dev, graph=graph)
            np.testing.assert_array_equal(t_tp, t_ref)
            np.testing.assert_array_equal(l_tp, l_ref)
            if run.xchg is not None:
                run.xchg.close()
            del run
        run = TP.W8A8TPLlamaRunner.from_package(pkg_dir, device=dev, num_blocks=len(lengths) * per_seq,
                                                block_size=bs)
        t_tp, l_tp = _generate(run, prompts, bt, 5, dev, graph=True)
        np.testing.assert_array_equal(t_tp, t_ref)
        np.testing.assert_array_equal(l_tp, l_ref)
        del run
        _lib.device_status()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # reported by the parent
        import traceback
        errors.put(f"rank {rank}: {e!r}\n{traceback.format_exc()}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_bit_identical_to_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    from oracle import w8a8 as O
    from nanopointllm_b200 import package as P, synthetic as S

    class OracleWeights:  # the package's int8 weights, quantised on the host
        def __init__(self, sd):
            self.sd = sd

        def linear(self, module):
            q, s = O.per_output_weight_quant(self.sd[module + ".weight"].float().numpy())
            return torch.from_numpy(q), torch.from_numpy(s.reshape(-1))

        def dense(self, name):
            return self.sd[name]

    P.write_w8a8_llama_package(tmp_path, S.TINY, OracleWeights(S.llama_weights(S.TINY, seed=0)))
    world = 2
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path), errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=400)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not msgs, "\n".join(msgs)
    assert all(p.exitcode == 0 for p in procs)
