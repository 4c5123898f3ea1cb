"""Continuous-batching decode driver over the W8A8 runner, and the
data-parallel request router across replicas.

The per-replica loop follows the reference's engine (nanopointllm/engine):
  sequence.py:10-80        a request's state (token ids, block table, status)
  block_manager.py:67-160  paged KV blocks: allocate a prompt's blocks at
                           admission, one more when the last token starts a
                           block, free them when the sequence ends or is
                           preempted (no prefix cache: prompts carry point
                           embeddings, which the reference never shares)
  scheduler.py:46-127      FIFO two-queue scheduling: admit waiting prompts
                           first (token budget, sequence limit, free blocks),
                           decode every other running sequence, preempt (and
                           later recompute) a sequence that cannot get a block
  llm_engine.py:116-122    one step = schedule, run the mixed batch, append
                           the sampled tokens
Steps with prompts run eagerly through the runner (prefill rows through the
varlen prefill attention, decode rows through the decode kernel); decode-only
steps replay a strict CUDA graph per batch bucket (runner.DecodeGraph), with
padding rows at slot -1 and context length 0.

Data parallel: ``route`` splits a request list over the replicas (longest
expected work first, each to the least-loaded replica); every rank runs its
share on its own GPU and ``gather_metrics`` combines the per-rank results on
rank 0 (torch.distributed, no collective inside a step).
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Callable, Optional, Sequence as Seq

import torch
import torch.nn.functional as F


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


@dataclass
class Request:
    """One serving request: ``n_point_rows`` point-feature embedding rows
    (the encoded point cloud, placed before the text), then the text token
    ids; generate ``max_tokens`` tokens greedily."""
    rid: int
    text_ids: list[int]
    max_tokens: int
    n_point_rows: int = 0
    point_seed: int = 0


class Sequence:
    """A request being served (sequence.py:17-80). Positions 0..n_point_rows-1
    hold the point rows, then the text ids, then the generated ids."""

    def __init__(self, req: Request):
        self.req = req
        self.token_ids: list[int] = list(req.text_ids)
        self.num_prompt_tokens = req.n_point_rows + len(req.text_ids)
        self.status = SequenceStatus.WAITING
        self.block_table: list[int] = []
        self.t_first_token: Optional[float] = None
        self.t_done: Optional[float] = None
        self.preemptions = 0

    @property
    def num_tokens(self) -> int:
        return self.req.n_point_rows + len(self.token_ids)

    @property
    def num_completion_tokens(self) -> int:
        return self.num_tokens - self.num_prompt_tokens

    @property
    def output_ids(self) -> list[int]:
        return self.token_ids[len(self.req.text_ids):]

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]


class BlockManager:
    """Paged KV blocks of one replica (block_manager.py:34-160, without the
    prefix cache)."""

    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free: deque[int] = deque(range(num_blocks))

    @property
    def num_free(self) -> int:
        return len(self.free)

    def blocks_for(self, seq: Sequence) -> int:
        return (seq.num_tokens + self.block_size - 1) // self.block_size

    def can_allocate(self, seq: Sequence) -> bool:
        return self.num_free >= self.blocks_for(seq)

    def allocate(self, seq: Sequence) -> None:
        if seq.block_table:
            raise RuntimeError("sequence already holds blocks")
        n = self.blocks_for(seq)
        if n > self.num_free:
            raise RuntimeError("not enough free KV blocks")
        seq.block_table = [self.free.popleft() for _ in range(n)]

    def deallocate(self, seq: Sequence) -> None:
        self.free.extend(reversed(seq.block_table))
        seq.block_table = []

    def can_append(self, seq: Sequence) -> bool:
        """The next decode writes the KV of the last token; it needs a new
        block when that token is the first of one (block_manager.py:133-141)."""
        return seq.num_tokens % self.block_size != 1 or self.num_free >= 1

    def may_append(self, seq: Sequence) -> None:
        if seq.num_tokens % self.block_size == 1:
            if not self.free:
                raise RuntimeError("no free KV block to append")
            seq.block_table.append(self.free.popleft())


class Scheduler:
    """FIFO two-queue scheduler (scheduler.py:46-127): prompts first, then
    every other running sequence decodes."""

    def __init__(self, max_num_seqs: int, max_num_batched_tokens: int, block_manager: BlockManager,
                 eos_token_id: Optional[int] = None):
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.bm = block_manager
        self.eos_token_id = eos_token_id
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []

    def add(self, seq: Sequence) -> None:
        self.waiting.append(seq)

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def preempt(self, seq: Sequence) -> None:
        """Back to the front of the queue; its blocks are freed and its whole
        sequence (prompt + tokens so far) is prefilled again later."""
        seq.status = SequenceStatus.WAITING
        seq.preemptions += 1
        self.bm.deallocate(seq)
        if seq in self.running:
            self.running.remove(seq)
        self.waiting.appendleft(seq)

    def schedule(self) -> tuple[list[Sequence], list[Sequence]]:
        prefill: list[Sequence] = []
        budget = 0
        while self.waiting:
            seq = self.waiting[0]
            if len(self.running) >= self.max_num_seqs or not self.bm.can_allocate(seq):
                break
            if budget + seq.num_tokens > self.max_num_batched_tokens and prefill:
                break
            budget += seq.num_tokens
            self.waiting.popleft()
            self.bm.allocate(seq)
            seq.status = SequenceStatus.RUNNING
            self.running.append(seq)
            prefill.append(seq)
        admitted = {id(s) for s in prefill}
        decode: list[Sequence] = []
        for seq in [s for s in self.running if id(s) not in admitted]:
            if self.bm.can_append(seq):
                self.bm.may_append(seq)
                decode.append(seq)
            else:
                self.preempt(seq)
        return prefill, decode

    def postprocess(self, seqs: Seq[Sequence], tokens: Seq[int], now: float) -> list[Sequence]:
        """Appends each sampled token; returns the sequences that finished."""
        done = []
        for seq, tok in zip(seqs, tokens):
            seq.token_ids.append(int(tok))
            if seq.t_first_token is None:
                seq.t_first_token = now
            if seq.num_completion_tokens >= seq.req.max_tokens or (
                    self.eos_token_id is not None and int(tok) == self.eos_token_id):
                seq.status = SequenceStatus.FINISHED
                seq.t_done = now
                self.bm.deallocate(seq)
                self.running.remove(seq)
                done.append(seq)
        return done


DECODE_BUCKETS = (1, 2, 4, 8, 16, 32, 64)


class ServingEngine:
    """One replica: a W8A8LlamaRunner (on its own KV pool), a block manager
    and a scheduler. ``run(requests)`` serves them to completion."""

    def __init__(self, runner, *, max_num_seqs: int = 64, max_num_batched_tokens: int = 16384,
                 max_blocks_per_seq: int, eos_token_id: Optional[int] = None, use_graphs: bool = True,
                 point_rows_fn: Optional[Callable[[Request], torch.Tensor]] = None):
        from . import runner as R
        self.R = R
        self.runner = runner
        self.bm = BlockManager(runner.num_blocks, runner.block_size)
        self.sched = Scheduler(max_num_seqs, max_num_batched_tokens, self.bm, eos_token_id)
        self.max_blocks = max_blocks_per_seq
        self.use_graphs = use_graphs
        self.graphs: dict[int, object] = {}
        self.point_rows_fn = point_rows_fn or self._default_point_rows
        self.steps = {"mixed": 0, "decode": 0}
        self.step_s = {"mixed": 0.0, "decode": 0.0}  # host wall time per step kind (each step ends synchronised)

    def _default_point_rows(self, req: Request) -> torch.Tensor:
        """Seeded N(0, 1) point-feature rows standing in for the point encoder's output."""
        g = torch.Generator(device=self.runner.device).manual_seed(req.point_seed)
        return torch.randn(req.n_point_rows, self.runner.shape.hidden, generator=g,
                           device=self.runner.device).half()

    def _slots(self, seq: Sequence, positions: range) -> list[int]:
        bs = self.bm.block_size
        return [seq.block_table[p // bs] * bs + p % bs for p in positions]

    def _block_tables(self, seqs: Seq[Sequence], rows: int) -> torch.Tensor:
        """int32 [rows, max_blocks] (host): each sequence's blocks, zero-padded;
        rows past the sequences are zero. Built as one list (a per-element
        tensor write costs microseconds each on the host)."""
        w = self.max_blocks
        table = []
        for s in seqs:
            if len(s.block_table) > w:
                raise RuntimeError(f"request {s.req.rid} needs more than {w} KV blocks")
            table.append(s.block_table + [0] * (w - len(s.block_table)))
        table.extend([[0] * w for _ in range(rows - len(seqs))])
        return torch.tensor(table, dtype=torch.int32).reshape(rows, w)

    def _decode_metadata(self, decode: Seq[Sequence], bucket: int):
        """Host tensors of a decode step padded to `bucket` rows: token ids,
        positions, slots (-1 for padding rows), context lengths and block
        tables (paged_model_runner.py:332-383 prepare_decode)."""
        pad = bucket - len(decode)
        bs = self.bm.block_size
        last = [s.num_tokens - 1 for s in decode]
        ids = torch.tensor([s.last_token for s in decode] + [0] * pad, dtype=torch.long)
        pos = torch.tensor(last + [0] * pad, dtype=torch.long)
        slots = torch.tensor([s.block_table[p // bs] * bs + p % bs for s, p in zip(decode, last)] + [-1] * pad,
                             dtype=torch.int32)
        ctx = torch.tensor([p + 1 for p in last] + [0] * pad, dtype=torch.int32)
        return ids, pos, slots, ctx, self._block_tables(decode, bucket)

    def _run_mixed(self, prefill: list[Sequence], decode: list[Sequence]) -> list[int]:
        """Prompts (their whole sequence) and decode rows in one eager forward
        (paged_model_runner.py:386-504 run_mixed)."""
        r, dev = self.runner, self.runner.device
        rows, positions, slots, seq_lens, ctx = [], [], [], [], []
        for s in prefill:
            ids = torch.tensor(s.token_ids, dtype=torch.long, device=dev)
            text = F.embedding(ids, r.embed)
            rows.append(torch.cat([self.point_rows_fn(s.req), text]) if s.req.n_point_rows else text)
            positions.extend(range(s.num_tokens))
            slots.extend(self._slots(s, range(s.num_tokens)))
            seq_lens.append(s.num_tokens)
            ctx.append(s.num_tokens)
        if decode:  # one embedding lookup for all decode rows
            rows.append(F.embedding(torch.tensor([s.last_token for s in decode], device=dev), r.embed))
        for s in decode:
            positions.append(s.num_tokens - 1)
            slots.extend(self._slots(s, range(s.num_tokens - 1, s.num_tokens)))
            seq_lens.append(1)
            ctx.append(s.num_tokens)
        seqs = prefill + decode
        pos = torch.tensor(positions, dtype=torch.long, device=dev)
        self.R.set_forward_context(self.R.ForwardContext(
            slot_mapping=torch.tensor(slots, dtype=torch.int32, device=dev),
            block_tables=self._block_tables(seqs, len(seqs)).to(dev),
            context_lens=torch.tensor(ctx, dtype=torch.int32, device=dev), position_ids=pos, seq_lens=seq_lens))
        try:
            logits = r.forward(inputs_embeds=torch.cat(rows), position_ids=pos, last_only=True)
        finally:
            self.R.clear_forward_context()
        self.steps["mixed"] += 1
        return logits[0].argmax(-1).tolist()

    def _run_decode(self, decode: list[Sequence]) -> list[int]:
        n = len(decode)
        bucket = next((b for b in DECODE_BUCKETS if b >= n), None)
        if not self.use_graphs or bucket is None:
            return self._run_mixed([], decode)
        dg = self.graphs.get(bucket)
        if dg is None:
            dg = self.graphs[bucket] = self.R.DecodeGraph(self.runner, bucket, self.max_blocks)
        ids, pos, slots, ctx, bt = self._decode_metadata(decode, bucket)
        if dg.graph is None:
            dg.load(ids, pos, slots, ctx, bt, non_blocking=False)
            dg.capture()  # runs the step twice eagerly: the KV writes are the same values
        dg.load(ids, pos, slots, ctx, bt, non_blocking=False)
        self.steps["decode"] += 1
        return dg.replay()[:n].tolist()

    def step(self) -> list[Sequence]:
        prefill, decode = self.sched.schedule()
        if not prefill and not decode:
            if self.sched.waiting:
                raise RuntimeError("a waiting request does not fit in the KV pool")
            return []
        t0 = time.perf_counter()
        tokens = self._run_mixed(prefill, decode) if prefill else self._run_decode(decode)
        now = time.perf_counter()
        self.step_s["mixed" if prefill else "decode"] += now - t0
        return self.sched.postprocess(prefill + decode, tokens, now)

    def run(self, requests: Seq[Request]) -> dict:
        """Serves every request; returns per-request outputs and timings."""
        seqs = [Sequence(q) for q in requests]
        for s in seqs:
            self.sched.add(s)
        torch.cuda.synchronize(self.runner.device)
        t0 = time.perf_counter()
        while not self.sched.is_finished():
            self.step()
        torch.cuda.synchronize(self.runner.device)
        t1 = time.perf_counter()
        if self.bm.num_free != self.bm.num_blocks:
            raise RuntimeError("KV blocks leaked")
        return {
            "outputs": {s.req.rid: s.output_ids for s in seqs},
            "ttft_s": {s.req.rid: s.t_first_token - t0 for s in seqs},
            "elapsed_s": t1 - t0,
            "output_tokens": sum(len(s.output_ids) for s in seqs),
            "prompt_tokens": sum(s.num_prompt_tokens for s in seqs),
            "preemptions": sum(s.preemptions for s in seqs),
            "steps": dict(self.steps),
            "step_s": {k: round(v, 4) for k, v in self.step_s.items()},
        }


# ---------------------------------------------------------------- data parallel
def route(requests: Seq[Request], world: int) -> list[list[Request]]:
    """Longest expected work first, each request to the replica with the least
    work so far (prompt + output tokens; ties to the lower rank)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    shares: list[list[Request]] = [[] for _ in range(world)]
    load = [0] * world
    order = sorted(requests, key=lambda q: (-(q.n_point_rows + len(q.text_ids) + q.max_tokens), q.rid))
    for q in order:
        r = min(range(world), key=lambda i: (load[i], i))
        shares[r].append(q)
        load[r] += q.n_point_rows + len(q.text_ids) + q.max_tokens
    for s in shares:
        s.sort(key=lambda q: q.rid)  # each replica serves its share in arrival order
    return shares


def gather_metrics(result: dict, group=None) -> Optional[dict]:
    """Combines the replicas' results on rank 0 (None on the other ranks):
    output tokens of all replicas over the slowest replica's time."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts: list = [None] * world if dist.get_rank(group) == 0 else None
    mine = {k: result[k] for k in ("elapsed_s", "output_tokens", "prompt_tokens", "preemptions", "ttft_s")}
    dist.gather_object(mine, parts, dst=0, group=group)
    if parts is None:
        return None
    elapsed = max(p["elapsed_s"] for p in parts)
    tokens = sum(p["output_tokens"] for p in parts)
    ttft = sorted(v for p in parts for v in p["ttft_s"].values())

    def pct(q):
        return ttft[min(len(ttft) - 1, int(q * len(ttft)))] if ttft else None

    return {"replicas": world, "output_tokens": tokens, "prompt_tokens": sum(p["prompt_tokens"] for p in parts),
            "elapsed_s": elapsed, "output_tokens_per_s": tokens / elapsed if elapsed > 0 else None,
            "ttft_p50_s": pct(0.5), "ttft_p99_s": pct(0.99),
            "preemptions": sum(p["preemptions"] for p in parts),
            "per_replica_elapsed_s": [p["elapsed_s"] for p in parts]}


def gather_metrics_local(result: dict) -> dict:
    """gather_metrics for a single replica (no process group)."""
    ttft = sorted(result["ttft_s"].values())
    pct = (lambda q: ttft[min(len(ttft) - 1, int(q * len(ttft)))] if ttft else None)
    e = result["elapsed_s"]
    return {"replicas": 1, "output_tokens": result["output_tokens"], "prompt_tokens": result["prompt_tokens"],
            "elapsed_s": e, "output_tokens_per_s": result["output_tokens"] / e if e > 0 else None,
            "ttft_p50_s": pct(0.5), "ttft_p99_s": pct(0.99), "preemptions": result["preemptions"],
            "per_replica_elapsed_s": [e]}


def config5_requests(n: int = 256, *, vocab: int, seed: int = 5, n_point_rows: int = 513,
                     text_range: tuple[int, int] = (47, 511), outputs: tuple[int, ...] = (16, 64, 256)) -> list[Request]:
    """Config 5's synthetic workload: every request has 513 point-embedding
    rows, a uniform U{47..511} text length with uniform token ids, and an
    output length drawn from {16, 64, 256}; all arrive at t = 0."""
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for i in range(n):
        t_len = int(torch.randint(text_range[0], text_range[1] + 1, (1,), generator=g))
        out = outputs[int(torch.randint(0, len(outputs), (1,), generator=g))]
        ids = torch.randint(0, vocab, (t_len,), generator=g).tolist()
        reqs.append(Request(rid=i, text_ids=ids, max_tokens=out, n_point_rows=n_point_rows, point_seed=seed * 100003 + i))
    return reqs
