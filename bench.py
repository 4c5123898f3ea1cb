"""Benchmark: W8A8 decode tokens/s of a Llama-7B-architecture backbone at
batch 8 and 1024-token context on B200, through libnpl_w8a8.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: random-init 7B W8A8 (32 layers, hidden 4096, 32
heads x 128, intermediate 11008, vocab 32003), batch 8, each sequence 513
point-embedding rows ~N(0,1) + 511 text tokens (uniform ids) = 1024-token
context prefilled through the same W8A8 runner, fp16 paged KV pool with
block_size 256 and a randomly permuted block table, greedy decode. A step is
one full decode step (32 layers + LM head + argmax) for the 8 sequences,
replayed as one CUDA graph; ``value`` = 8 * N * K / max-over-ranks time.

Every step streams 6.6 GB of int8 weights and ~4.3 GB of fp16 KV, both far
larger than the 126 MB L2, so no L2 flush is inserted between steps.

``e2e`` measures the same steps through the runner's public API the way a
serving loop drives it: each step copies its metadata (token ids, positions,
slots, context lengths, block tables) from pinned host memory to the device,
replays the graph and reads the 8 greedy tokens back to the host.

With --gpus N (torchrun, one process per GPU) every rank runs an independent
replica on its own requests (data parallel, no collective in the step).

``--kernel-case NAME`` runs one op of the step alone (``--warmup`` eager
launches, then ``--steps`` launches captured in a CUDA graph and replayed
twice) on synthetic data of the config-3 / config-4 shapes and prints its
per-launch device time and algorithmic throughput; it is the command the ncu
summaries in profiles/ are taken with. Cases: qkv, o, gate_up,
down, lm_head (decode linears, M = 8), attention (B = 8, context 1040),
rmsnorm_quant, prefill (the five config-4 GEMMs at M = 4480), int8_peak
(cuBLASLt int8 GEMM through torch._int_mm, 8192^3: the measured int8 tensor
peak the prefill roofline is reported against), prefill_attention (the
varlen prefill attention at config 4: 8 x 560 tokens, causal FLOP/s against
the measured dense fp16/bf16 peak), package_load (start-up of
a 7B-geometry runner with ``--layers`` layers from fp16 host weights against
from the checksummed int8 package), prefill_forward (one eager prefill
forward over ``--prefill-seqs`` x ``--prefill-len`` tokens, whole and per op).

``--impl reference`` times the reference's CPU W8A8 decode path on the host
cores: oracle/cpu_decode.py, a torch restatement of it (the reference itself
is Python code that is not on the GPU box) with the int32 matmuls of
integer_linear_per_output_reference. Each bench step is one of the 32
decoder layers (all cost the same); the value is the full step's tokens/s.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import pathlib
import statistics
import sys
import time

REPO = pathlib.Path(__file__).resolve().parent
METRIC = "W8A8 decode tokens/s (7B, bs=8, ctx 1024); int8-linear % of HBM roofline"
BATCH = 8
CTX = 1024
POINT_TOKENS = 513
BLOCK_SIZE = 256


def _register_package() -> None:
    if "nanopointllm_b200" in sys.modules:
        return
    pkg = REPO / "nano-pointllm_b200"
    spec = importlib.util.spec_from_file_location(
        "nanopointllm_b200", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["nanopointllm_b200"] = mod
    spec.loader.exec_module(mod)


def _peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and throttle reasons sampled every 10 ms through NVML while the
    timed region runs (reading only; no setting is changed)."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples: list[tuple[int, int, int]] = []
        self._stop = None
        self._thread = None
        self.error = None

    def _run(self):
        import pynvml
        try:
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self._stop.is_set():
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((sm, smax, reasons))
                self._stop.wait(0.01)
        except Exception as e:  # noqa: BLE001 - report, do not fail the bench
            self.error = repr(e)

    def start(self):
        import threading
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        self._stop.set()
        self._thread.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"no samples: {self.error}"]}
        reasons = set()
        for _, _, r in self.samples:
            for name, bit in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------- our arm
def build_runner(torch, shape, steps_total: int, device, seed: int, tp: bool = False, peer_exchange: bool = True):
    """The 7B W8A8 runner (tp: the tensor-parallel runner over all ranks of
    the default process group, every rank building from the same seed)."""
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    from nanopointllm_b200 import tp as TP
    blocks_per_seq = (CTX + steps_total + BLOCK_SIZE - 1) // BLOCK_SIZE
    num_blocks = BATCH * blocks_per_seq + 4
    weights = S.LazyLlamaWeights(shape, seed=seed, device=str(device))
    if tp:
        run = TP.W8A8TPLlamaRunner(shape, weights, device=device, num_blocks=num_blocks, block_size=BLOCK_SIZE,
                                   peer_exchange=peer_exchange)
    else:
        run = R.W8A8LlamaRunner(shape, weights, device=device, num_blocks=num_blocks, block_size=BLOCK_SIZE)
    bt = S.permuted_block_tables(BATCH, blocks_per_seq, num_blocks, seed=seed + 3).to(device)
    return run, bt


def prefill(torch, run, bt, device, seed: int):
    """1024-token contexts: 513 point embeddings ~N(0,1) + 511 text tokens."""
    from nanopointllm_b200 import runner as R
    shape = run.shape
    g = torch.Generator(device=device).manual_seed(seed + 7)
    points = torch.randn(BATCH, POINT_TOKENS, shape.hidden, generator=g, device=device).half()
    text = torch.randint(0, shape.vocab, (BATCH, CTX - POINT_TOKENS), generator=g, device=device)
    emb = torch.cat([points, torch.nn.functional.embedding(text, run.embed)], dim=1).reshape(-1, shape.hidden)
    pos = torch.arange(CTX, device=device).repeat(BATCH)
    blk = torch.arange(CTX, device=device) // BLOCK_SIZE
    off = torch.arange(CTX, device=device) % BLOCK_SIZE
    slots = (bt[:, blk].long() * BLOCK_SIZE + off).reshape(-1).to(torch.int32)
    R.set_forward_context(R.ForwardContext(
        slot_mapping=slots, block_tables=bt, context_lens=torch.full((BATCH,), CTX, dtype=torch.int32, device=device),
        position_ids=pos, seq_lens=[CTX] * BATCH))
    try:
        logits = run.forward(inputs_embeds=emb, position_ids=pos, last_only=True)
    finally:
        R.clear_forward_context()
    return logits[0].argmax(-1)


def step_metadata(torch, bt, step: int, device):
    """Metadata of decode step `step` (0-based): the new token sits at
    position CTX + step."""
    p = CTX + step
    positions = torch.full((BATCH,), p, dtype=torch.int64, device=device)
    slots = (bt[:, p // BLOCK_SIZE].long() * BLOCK_SIZE + p % BLOCK_SIZE).to(torch.int32)
    ctx = torch.full((BATCH,), p + 1, dtype=torch.int32, device=device)
    return positions, slots, ctx


# ------------------------------------------------------------- multi-rank
def rank_seed(rank: int) -> int:
    """Each data-parallel replica serves its own synthetic requests."""
    return 1000 * rank


def max_over_ranks(torch, dist, value: float, device) -> float:
    """A time measured on every rank -> the slowest rank's (the whole job is
    done when the last replica is done). Identity without a process group."""
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def linear_bytes(m: int, n: int, k: int, out_cols: int, residual: bool, fp16_x: bool) -> int:
    """Algorithmic bytes of one W8A8 linear launch: int8 weight + fp32 weight
    scales + activations (int8 + fp32 scales, or fp16 rows when the
    quantisation is fused in) + fp16 output (+ fp16 residual read)."""
    x = 2 * m * k if fp16_x else m * k + 4 * m
    return n * k + 4 * n + x + 2 * m * out_cols + (2 * m * out_cols if residual else 0)


def measured_traffic() -> dict[str, int]:
    """DRAM bytes (read + write) per launch of each decode-step kernel, from
    the committed ncu summary profiles/decode_step_traffic.md (one capture of
    each kernel alone on the config-3 shapes): op name -> bytes."""
    out = {}
    path = REPO / "profiles" / "decode_step_traffic.md"
    for line in path.read_text().splitlines():
        cells = [c.strip() for c in line.strip().strip("|").split("|")]
        if len(cells) == 4 and cells[2].isdigit():
            out[cells[0]] = int(cells[2])
    return out


def op_bytes(shape, name: str, ctx_len: int, fused_mlp: bool = False) -> int:
    m, h, i_, v = BATCH, shape.hidden, shape.intermediate, shape.vocab
    qkv_n = (shape.heads + 2 * shape.kv_heads) * shape.head_dim
    if name == "linear.qkv":  # q out, k/v written to the cache (+ positions, slots, cos/sin rows)
        return linear_bytes(m, qkv_n, h, qkv_n, False, False)
    if name == "linear.o":
        return linear_bytes(m, h, shape.heads * shape.head_dim, h, True, False)
    if name == "linear.gate_up":
        return linear_bytes(m, 2 * i_, h, i_, False, False)
    if name == "linear.down":  # fused: fp16 input rows, quantised in the kernel
        return linear_bytes(m, h, i_, h, True, fused_mlp)
    if name == "linear.lm_head":
        return linear_bytes(m, v, h, v, False, False)
    if name == "attention":
        # fp16 K and V of every context token of every head, q in, out
        return m * ctx_len * shape.kv_heads * shape.head_dim * 2 * 2 + 2 * 2 * m * shape.heads * shape.head_dim
    return 0


def bench_shape(args):
    from nanopointllm_b200 import synthetic as S
    return S.LLAMA_7B if args.layers == 32 else S.LlamaShape(**{**S.LLAMA_7B.as_dict(), "layers": args.layers})


def timed_decode(args, torch, dist, run, bt, first, device, steps_total: int):
    """Captures the decode graph, runs the warm-up steps, then times
    args.steps replays on the device (max over ranks) and args.steps replays
    end to end (pinned host metadata in, greedy tokens out). Returns the
    graph, the next step index, the device and e2e times (ms), the
    per-step host<->device bytes and the clock record."""
    from nanopointllm_b200 import runner as R
    graph = R.DecodeGraph(run, BATCH, bt.shape[1])
    step = 0
    positions, slots, ctx = step_metadata(torch, bt, step, device)
    graph.load(first, positions, slots, ctx, bt)
    graph.capture()

    # device-resident metadata of every step, prepared before timing
    meta = [step_metadata(torch, bt, s, device) for s in range(steps_total)]

    def device_step(s: int):
        positions, slots, ctx = meta[s]
        graph.positions.copy_(positions)
        graph.slots.copy_(slots)
        graph.context_lens.copy_(ctx)
        tok = graph.replay()
        graph.ids.copy_(tok)
        return tok

    for _ in range(args.warmup):
        device_step(step)
        step += 1
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(int(visible.split(",")[torch.cuda.current_device()]) if visible
                          else torch.cuda.current_device())
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        device_step(step)
        step += 1
    e1.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    dev_ms = max_over_ranks(torch, dist, e0.elapsed_time(e1), device)
    if dist is not None:
        dist.barrier()

    # ---- e2e: host metadata in (pinned), graph replay, tokens out to host
    pin = lambda x: x.cpu().pin_memory()
    host_meta = [tuple(pin(x) for x in meta[step + i]) for i in range(args.steps)]
    host_bt = pin(bt)
    host_ids = pin(graph.ids)
    host_out = torch.empty(BATCH, dtype=torch.int64).pin_memory()
    h2d = d2h = 0
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(args.steps):
        positions, slots, ctx = host_meta[i]
        graph.load(host_ids, positions, slots, ctx, host_bt, non_blocking=True)
        tok = graph.replay()
        host_out.copy_(tok, non_blocking=True)
        stream.synchronize()
        host_ids.copy_(host_out)
        h2d = sum(x.numel() * x.element_size() for x in (host_ids, positions, slots, ctx, host_bt))
        d2h = host_out.numel() * host_out.element_size()
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, e2.elapsed_time(e3), device)
    step += args.steps
    return graph, step, meta, dev_ms, e2e_ms, h2d, d2h, clock_info


def run_ours(args, torch, dist, rank: int, world: int, device) -> dict | None:
    from nanopointllm_b200 import _lib, runner as R
    shape = bench_shape(args)
    n_eager = 2
    steps_total = args.warmup + args.steps * 2 + n_eager + 2
    run, bt = build_runner(torch, shape, steps_total, device, seed=rank_seed(rank))
    first = prefill(torch, run, bt, device, seed=rank_seed(rank))
    torch.cuda.synchronize()
    graph, step, meta, dev_ms, e2e_ms, h2d, d2h, clock_info = timed_decode(args, torch, dist, run, bt, first,
                                                                           device, steps_total)

    # ---- per-kernel device time: a second decode graph whose ops are each
    # bracketed by timing events recorded inside the graph (on the launch
    # stream), replayed like the timed graph
    records: list[tuple[str, object, object]] = []

    def timer(name, fn, *a, **kw):
        s0 = torch.cuda.Event(enable_timing=True, external=True)
        s1 = torch.cuda.Event(enable_timing=True, external=True)
        s0.record()
        out = fn(*a, **kw)
        s1.record()
        records.append((name, s0, s1))
        return out

    ctx_mid = CTX + step
    pgraph = R.DecodeGraph(run, BATCH, bt.shape[1])
    positions, slots, ctx = meta[step]
    pgraph.load(graph.ids, positions, slots, ctx, bt)
    run.timer = timer
    try:
        pgraph.capture()
    finally:
        run.timer = None
    n_warm_rec = len(records) - len(records) // 3  # capture() runs the step twice before recording it
    records = records[n_warm_rec:]
    per_op: dict[str, list[float]] = {}
    for _ in range(n_eager):
        positions, slots, ctx = meta[step]
        pgraph.load(graph.ids, positions, slots, ctx, bt)
        pgraph.replay()
        torch.cuda.synchronize()
        for name, s0, s1 in records:
            per_op.setdefault(name, []).append(s0.elapsed_time(s1))
        step += 1
    del pgraph
    _lib.device_status()

    standalone = standalone_linears(torch, run, shape, device) if rank == 0 else {}
    if rank != 0:
        return None
    peak, peak_kind = _peaks()
    for v in standalone.values():
        v["frac"] = round(v["gbs"] / peak, 4)
    lin_names = [n for n in per_op if n.startswith("linear.")]
    # The bracketing events serialise the step (no programmatic-dependent-
    # launch overlap), so the bracketed op times add up to more than the
    # measured step. Each op's in-step time is its bracketed time scaled by
    # (measured step / bracketed step): the apportioned times add up to
    # ms_per_step exactly.
    step_ms = dev_ms / args.steps
    bracketed_step_ms = sum(sum(t) for t in per_op.values()) / n_eager
    share_scale = step_ms / bracketed_step_ms
    lin_ms = sum(sum(per_op[n]) for n in lin_names)
    fused = run.fuse_mlp_quant
    lin_bytes = sum(op_bytes(shape, n, ctx_mid, fused) * len(per_op[n]) for n in lin_names)
    lin_launches = sum(len(per_op[n]) for n in lin_names)
    achieved = lin_bytes / (lin_ms * share_scale * 1e-3) / 1e9
    achieved_bracketed = lin_bytes / (lin_ms * 1e-3) / 1e9
    traffic_table = measured_traffic()
    traffic = sum(traffic_table[n] * len(per_op[n]) for n in lin_names) / max(1, lin_launches)
    kernels = {}
    for name, times in per_op.items():
        b = op_bytes(shape, name, ctx_mid, fused)
        avg = sum(times) / len(times)
        kernels[name] = {"launches_per_step": len(times) // n_eager, "avg_us_bracketed": round(avg * 1e3, 2),
                         "avg_us_in_step": round(avg * share_scale * 1e3, 2), "share": None}
        if b:
            kernels[name]["gbs_in_step"] = round(b / (avg * share_scale * 1e-3) / 1e9, 1)
            kernels[name]["frac_in_step"] = round(b / (avg * share_scale * 1e-3) / 1e9 / peak, 4)
        if name in traffic_table:
            kernels[name]["traffic_per_launch"] = traffic_table[name]
    tot = sum(sum(t) for t in per_op.values())
    for name, times in per_op.items():
        kernels[name]["share"] = round(sum(times) / tot, 4)
    step_bytes = sum(op_bytes(shape, n, ctx_mid, fused) * len(t) for n, t in per_op.items()) / n_eager

    launches_per_step = sum(len(t) for t in per_op.values()) // n_eager  # every op is one library kernel
    tokens = BATCH * world * args.steps
    value = tokens / (dev_ms * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (W8A8: int8 x int8 -> int32, fp16 activations/KV)",
        "data": "synthetic (random-init 7B weights ~N(0,0.02); 513 point embeddings ~N(0,1) + 511 uniform text ids)",
        "config": {"workload": "config3: W8A8 Llama-7B-arch decode step, batch 8, ctx 1024 (prefilled), "
                               "block_size 256, permuted block table, greedy, CUDA graph",
                   "batch_per_gpu": BATCH, "context": CTX, "layers": shape.layers,
                   "parallelism": f"dp{world} (independent replicas)",
                   "l2": "no flush: each step streams 6.6 GB int8 weights + ~4.3 GB fp16 KV (>> 126 MB L2)"},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 2), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "kernel": "w8a8_linear_kernel (all 5 linears of the step)",
                     "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": round(traffic),
                     "traffic_unit": "DRAM bytes per launch (mean over the step's linear launches), from the ncu "
                                     "summary profiles/decode_step_traffic.md (dram__bytes_read.sum + "
                                     "dram__bytes_write.sum)",
                     "algorithmic_bytes_per_launch": round(lin_bytes / max(1, lin_launches)),
                     "algorithmic_bytes_per_step": lin_bytes // n_eager,
                     "launches_per_step": lin_launches // n_eager,
                     "timing": "each op bracketed by CUDA events recorded inside a copy of the decode graph, "
                               "replayed like the timed graph; the bracketed times (which serialise the "
                               "launches) are scaled so that the step's ops add up to the measured ms_per_step "
                               f"(scale {share_scale:.3f})",
                     "achieved_bracketed": round(achieved_bracketed, 1),
                     "frac_bracketed": round(achieved_bracketed / peak, 4),
                     "whole_step": {"algorithmic_bytes": round(step_bytes),
                                    "achieved": round(step_bytes / (step_ms * 1e-3) / 1e9, 1),
                                    "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / peak, 4),
                                    "note": "int8 weights + fp16 KV + activations of every op of the step over "
                                            "the measured ms_per_step"},
                     "standalone": standalone},
        "kernels": kernels,
        "clocks": clock_info,
    }
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(seconds=args.cpu_seconds)
    return line


def run_tp(args, torch, dist, rank: int, world: int, device) -> dict | None:
    """Config 3 with the tensor-parallel runner: ONE batch of 8 sequences
    split over the N ranks (heads and intermediate rows per rank, NCCL
    all-reduces after O and down, all-gathered logits), captured with its
    collectives in one decode graph per rank. Strong scaling: value =
    8 * K / max-over-ranks time."""
    from nanopointllm_b200 import _lib
    shape = bench_shape(args)
    steps_total = args.warmup + args.steps * 2 + 2
    run, bt = build_runner(torch, shape, steps_total, device, seed=0, tp=world > 1,
                           peer_exchange=not args.tp_nccl)
    first = prefill(torch, run, bt, device, seed=0)
    torch.cuda.synchronize()
    graph, step, meta, dev_ms, e2e_ms, h2d, d2h, clock_info = timed_decode(args, torch, dist, run, bt, first,
                                                                           device, steps_total)
    del graph  # releases the NCCL calls captured in it before the process group goes
    torch.cuda.synchronize()
    _lib.device_status()
    if rank != 0:
        return None
    tokens = BATCH * args.steps
    kernels_per_step = shape.layers * 9 + 2  # library kernels; NCCL collectives come on top
    return {
        "metric": METRIC, "value": round(tokens / (dev_ms * 1e-3), 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 (W8A8: int8 x int8 -> int32, fp16 activations/KV)",
        "data": "synthetic (random-init 7B weights ~N(0,0.02); 513 point embeddings ~N(0,1) + 511 uniform text ids)",
        "config": {"workload": "config3 decode step, tensor parallel: batch 8, ctx 1024 (prefilled), block_size "
                               "256, permuted block table, greedy, CUDA graph with the NCCL collectives",
                   "batch": BATCH, "context": CTX, "layers": shape.layers, "parallelism": f"tp{world}",
                   "exchanges_per_layer": ("absmax MAX + int32 SUM all-reduce before O and before down "
                                           "(4 NCCL all-reduces)" if args.tp_nccl or world == 1 else
                                           "absmax MAX (fused with the quantisation) and int32 SUM (fused "
                                           "with the dequant + residual) through NVLink peer memory, before "
                                           "O and before down (4 exchange kernels)") +
                                          "; logits all-gather (NCCL) once per step",
                   "l2": "no flush: each step streams the rank's weight and KV slices (>> 126 MB L2)"},
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 2), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": kernels_per_step * args.steps,
        "clocks": clock_info,
    }


def standalone_linears(torch, run, shape, device) -> dict:
    """Device time per launch of each decode linear over the step's own
    weights: one CUDA graph of the 32 layers' launches of that projection
    back to back (every weight read from DRAM), the activations fixed."""
    from nanopointllm_b200 import _lib as L, w8a8 as W
    g = torch.Generator(device=device).manual_seed(5)
    out = {}
    for name, attr, k, epi in (("linear.qkv", "qkv", shape.hidden, L.EPI_NONE),
                               ("linear.o", "o", shape.heads * shape.head_dim, L.EPI_RESIDUAL),
                               ("linear.gate_up", "gate_up", shape.hidden, L.EPI_SILU_MUL),
                               ("linear.down", "down", shape.intermediate, L.EPI_RESIDUAL)):
        lins = [getattr(layer, attr) for layer in run.layers]
        n = lins[0].out_features
        qa = torch.randint(-127, 128, (BATCH, k), dtype=torch.int8, device=device, generator=g)
        sa = torch.rand(BATCH, device=device, generator=g) * 1e-2
        res = torch.randn(BATCH, n, device=device, generator=g).half() if epi == L.EPI_RESIDUAL else None
        dst = torch.empty(BATCH, n // 2 if epi == L.EPI_SILU_MUL else n, dtype=torch.float16, device=device)

        def launches():
            for lin in lins:
                W.linear_q(qa, sa, lin.qweight, lin.wscale, epilogue=epi, residual=res, out=dst)
        launches()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            launches()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / len(lins)
        nbytes = op_bytes(shape, name, CTX, False)
        out[name] = {"us_per_launch": round(us, 2), "gbs": round(nbytes / us / 1e3, 1)}
        del graph
    return out


# ------------------------------------------------------------- CPU arm
def cpu_layers(n_layers: int, warmup: int, seconds: float | None = None) -> tuple[list[float], float, int]:
    """The reference's CPU W8A8 decode path (oracle.cpu_decode: torch CPU,
    int32 matmuls like integer_linear_per_output_reference) on the host cores:
    ``warmup`` untimed decoder layers, then ``n_layers`` timed ones (fewer if
    ``seconds`` runs out first), then the final norm + LM head once. Every
    decoder layer has the same work (7B widths, batch 8, context 1024).
    Returns (layer times s, LM-head time s, threads)."""
    import torch
    sys.path.insert(0, str(REPO))
    from oracle.cpu_decode import CpuDecodeLayer
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layer = CpuDecodeLayer(BATCH, CTX, BLOCK_SIZE)
    for _ in range(warmup):
        layer.layer(layer.x)
    layer.lm_head(layer.x)
    times = []
    t_end = None if seconds is None else time.perf_counter() + seconds
    for _ in range(n_layers):
        t0 = time.perf_counter()
        layer.layer(layer.x)
        times.append(time.perf_counter() - t0)
        if t_end is not None and time.perf_counter() > t_end:
            break
    t0 = time.perf_counter()
    layer.lm_head(layer.x)
    return times, time.perf_counter() - t0, threads


def cpu_step_seconds(times: list[float], head: float, layers: int = 32) -> float:
    """A full decode step of the 32-layer model from per-layer samples."""
    return layers * statistics.mean(times) + head


def cpu_baseline(seconds: float = 20.0) -> dict:
    """Reported beside our number: the reference's CPU decode path timed on
    a bounded sample (up to 20 decoder layers within ``seconds``, plus the LM
    head), scaled to a full 32-layer step."""
    times, head, threads = cpu_layers(20, 1, seconds)
    step_s = cpu_step_seconds(times, head)
    return {"value": round(BATCH / step_s, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} timed decoder layers (7B widths, batch 8, ctx 1024, paged KV) + the LM head "
                      f"on the host CPU: torch int32 matmuls as integer_linear_per_output_reference, SDPA "
                      f"attention; step = 32 x mean layer ({statistics.mean(times):.3f} s) + head ({head:.3f} s)",
            "s_per_step": round(step_s, 3)}


# ------------------------------------------------------- single-op cases
KERNEL_CASES = ("qkv", "o", "gate_up", "down", "lm_head", "attention", "rmsnorm_quant", "prefill", "int8_peak",
                "prefill_attention", "package_load", "prefill_forward")


def run_kernel_case(args, torch, device) -> dict:
    from nanopointllm_b200 import _lib as L, paged_attention as PA, runner as R, synthetic as S, w8a8 as W
    name = args.kernel_case
    g = torch.Generator(device=device).manual_seed(0)
    shape = S.LLAMA_7B
    h, inter, v = shape.hidden, shape.intermediate, shape.vocab
    qkv_n = (shape.heads + 2 * shape.kv_heads) * shape.head_dim

    def timed(fn, n_launch):
        """Device time per launch: the warm-up launches run eagerly, the timed
        ones are replayed back to back from a CUDA graph (no host gaps)."""
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (args.steps * n_launch)

    def weights(n, k):
        # enough distinct weight copies that consecutive launches miss L2
        copies = max(2, int(300e6 // (n * k)) + 1)
        return [torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=g) for _ in range(copies)]

    line = {"case": name}
    if name in ("qkv", "o", "gate_up", "down", "lm_head"):
        n, k, epi, res = {"qkv": (qkv_n, h, L.EPI_NONE, False), "o": (h, h, L.EPI_RESIDUAL, True),
                          "gate_up": (2 * inter, h, L.EPI_SILU_MUL, False),
                          "down": (h, inter, L.EPI_RESIDUAL, True), "lm_head": (v, h, L.EPI_NONE, False)}[name]
        ws = weights(n, k)
        sw = torch.rand(n, device=device, generator=g) * 1e-3
        qa = torch.randint(-127, 128, (BATCH, k), dtype=torch.int8, device=device, generator=g)
        sa = torch.rand(BATCH, device=device, generator=g) * 1e-2
        resid = torch.randn(BATCH, n, device=device, generator=g).half() if res else None
        out = torch.empty(BATCH, n // 2 if epi == L.EPI_SILU_MUL else n, dtype=torch.float16, device=device)
        us = timed(lambda i: W.linear_q(qa, sa, ws[i % len(ws)], sw, epilogue=epi, residual=resid, out=out), 1)
        nbytes = op_bytes(shape, "linear." + name, CTX, False)
        line.update({"kernel": "w8a8_linear_kernel", "shape": [BATCH, n, k], "us_per_launch": round(us, 2),
                     "algorithmic_bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1)})
    elif name == "attention":
        # config 3 by default (8 x 1040 tokens); --attn-batch / --attn-ctx LO HI
        # give serving-like batches with contexts drawn uniformly from [LO, HI]
        batch = args.attn_batch or BATCH
        lo, hi = args.attn_ctx or (CTX + 16, CTX + 16)
        ctx_l = torch.randint(lo, hi + 1, (batch,), generator=torch.Generator().manual_seed(1)).tolist()
        mb = (max(ctx_l) + BLOCK_SIZE - 1) // BLOCK_SIZE + 1
        nb = batch * mb
        sets = [(torch.randn(nb, BLOCK_SIZE, shape.kv_heads, shape.head_dim, device=device, generator=g).half(),
                 torch.randn(nb, BLOCK_SIZE, shape.kv_heads, shape.head_dim, device=device, generator=g).half())
                for _ in range(3)]
        bt = S.permuted_block_tables(batch, mb, nb, seed=1).to(device)
        q = torch.randn(batch, shape.heads, shape.head_dim, device=device, generator=g).half()
        cl = torch.tensor(ctx_l, dtype=torch.int32, device=device)
        q8 = torch.empty(batch, shape.heads * shape.head_dim, dtype=torch.int8, device=device)
        qs = torch.empty(batch, dtype=torch.float32, device=device)
        out = torch.empty_like(q)
        us = timed(lambda i: PA.paged_decode_attention(q, sets[i % 3][0], sets[i % 3][1], bt, cl, shape.head_dim ** -0.5,
                                                        1, out=out, quant_out=(q8, qs)), 1)
        nbytes = sum(op_bytes(shape, "attention", n) for n in ctx_l) // BATCH  # op_bytes counts BATCH sequences
        line.update({"kernel": "decode_attn_rows_kernel", "batch": batch,
                     "context": ctx_l[0] if lo == hi else [lo, hi], "us_per_launch": round(us, 2),
                     "algorithmic_bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1)})
    elif name == "rmsnorm_quant":
        x = torch.randn(BATCH, h, device=device, generator=g).half()
        w = torch.ones(h, device=device).half()
        us = timed(lambda i: R.rmsnorm_quant(x, w, 1e-6), 1)
        line.update({"kernel": "rmsnorm_quant_kernel", "shape": [BATCH, h], "us_per_launch": round(us, 2)})
    elif name == "prefill":
        m = 4480
        gemms = [("qkv", qkv_n, h), ("o", h, h), ("gate_up", 2 * inter, h), ("down", h, inter), ("lm_head", v, h)]
        xs = {k: torch.randint(-127, 128, (m, k), dtype=torch.int8, device=device, generator=g) for k in (h, inter)}
        sa = torch.rand(m, device=device, generator=g) * 1e-2
        wts = [(torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=g),
                torch.rand(n, device=device, generator=g) * 1e-3) for _, n, k in gemms]
        outs = [torch.empty(m, n, dtype=torch.float16, device=device) for _, n, _ in gemms]

        def all5(i):
            for (nm, n, k), (qw, sw), o in zip(gemms, wts, outs):
                W.linear_q(xs[k], sa, qw, sw, out=o)
        us = timed(all5, len(gemms))
        ops = sum(2 * m * n * k for _, n, k in gemms)
        t_step = us * len(gemms)
        line.update({"kernel": "w8a8_linear_kernel (NT = 256 tiles)", "config": "config4: M = 4480, the 5 GEMMs",
                     "us_per_5_gemms": round(t_step, 1), "tops": round(ops / t_step / 1e6, 1), "ops": ops})
    elif name == "int8_peak":
        n = 8192
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=device, generator=g)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=device, generator=g)
        us = timed(lambda i: torch._int_mm(a, b), 1)
        line.update({"kernel": "cuBLASLt int8 GEMM (torch._int_mm)", "shape": [n, n, n],
                     "us_per_launch": round(us, 1), "tops": round(2 * n ** 3 / us / 1e6, 1)})
    elif name == "prefill_attention":
        # config 4 by default: 8 prompts x 560 tokens prefilled in one step, 7B heads
        n_seq, q_len, bs = args.prefill_seqs, args.prefill_len, BLOCK_SIZE
        mb = -(-q_len // bs)
        nb = n_seq * mb
        k_cache = torch.randn(nb, bs, shape.kv_heads, shape.head_dim, device=device, generator=g).half()
        v_cache = torch.randn(nb, bs, shape.kv_heads, shape.head_dim, device=device, generator=g).half()
        bt = S.permuted_block_tables(n_seq, mb, nb, seed=1).to(device)
        q = torch.randn(n_seq * q_len, shape.heads, shape.head_dim, device=device, generator=g).half()
        lens = torch.full((n_seq,), q_len, dtype=torch.int32, device=device)
        offs = torch.arange(0, n_seq * q_len, q_len, dtype=torch.int32, device=device)
        out = torch.empty_like(q)
        us = timed(lambda i: PA.paged_varlen_attention(q, k_cache, v_cache, bt, lens, lens, offs,
                                                       shape.head_dim ** -0.5, 1, max_q_len=q_len, out=out), 1)
        pairs = n_seq * shape.heads * q_len * (q_len + 1) // 2   # causal (query, key) pairs
        flops = 4 * shape.head_dim * pairs                        # QK^T and P.V, 2 flops per MAC
        pf = REPO / "MEASURED_PEAKS.json"
        peak = float(json.loads(pf.read_text())["bf16_tflops"]) if pf.exists() else 1590.0
        line.update({"kernel": "prefill_attn_kernel<128> (tcgen05 kind::f16)",
                     "config": f"prefill: {n_seq} x {q_len} tokens, H = 32, D = 128, block_size 256"
                               + (" (config4)" if (n_seq, q_len) == (8, 560) else ""),
                     "us_per_launch": round(us, 2), "tflops": round(flops / us / 1e6, 1),
                     "causal_flops": flops, "peak_tflops": peak,
                     "peak_kind": "measured" if pf.exists() else "fallback",
                     "frac": round(flops / us / 1e6 / peak, 3)})
    elif name == "package_load":
        line.update(package_load_case(args, torch, device))
    elif name == "prefill_forward":
        line.update(prefill_forward_case(args, torch, device))
    L.device_status()
    return line


def prefill_forward_case(args, torch, device) -> dict:
    """One eager prefill forward of the 7B W8A8 runner (``--layers`` layers)
    over ``--prefill-seqs`` x ``--prefill-len`` tokens (the first mixed step
    of config-5 serving admits ~20 x 800): device time of the whole forward,
    then of every op bracketed by CUDA events (which stops programmatic
    dependent launch overlap, so the sum is slightly larger)."""
    import collections
    from nanopointllm_b200 import runner as R, synthetic as S
    shape = bench_shape(args)
    n_seq, t = args.prefill_seqs, args.prefill_len
    per = -(-t // BLOCK_SIZE)
    nb = n_seq * per + 4
    run = R.W8A8LlamaRunner(shape, S.LazyLlamaWeights(shape, seed=0, device=str(device)), device=device,
                            num_blocks=nb, block_size=BLOCK_SIZE)
    bt = S.permuted_block_tables(n_seq, per, nb, seed=3).to(device)
    g = torch.Generator(device=device).manual_seed(0)
    emb = torch.randn(n_seq * t, shape.hidden, generator=g, device=device).half()
    pos = torch.arange(t, device=device).repeat(n_seq)
    blk, off = torch.arange(t, device=device) // BLOCK_SIZE, torch.arange(t, device=device) % BLOCK_SIZE
    slots = (bt[:, blk].long() * BLOCK_SIZE + off).reshape(-1).to(torch.int32)
    ctx_lens = torch.full((n_seq,), t, dtype=torch.int32, device=device)

    def forward():
        R.set_forward_context(R.ForwardContext(slot_mapping=slots, block_tables=bt, context_lens=ctx_lens,
                                               position_ids=pos, seq_lens=[t] * n_seq))
        try:
            return run.forward(inputs_embeds=emb, position_ids=pos, last_only=True)
        finally:
            R.clear_forward_context()

    for _ in range(args.warmup):
        forward()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        forward()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    records = []

    def timer(name, fn, *a, **kw):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        out = fn(*a, **kw)
        s1.record()
        records.append((name, s0, s1))
        return out

    run.timer = timer
    forward()
    run.timer = None
    torch.cuda.synchronize()
    per_op: dict[str, float] = collections.OrderedDict()
    for n, a, b in records:
        per_op[n] = per_op.get(n, 0.0) + a.elapsed_time(b)
    return {"kernel": "whole prefill forward (eager)", "config": f"{n_seq} x {t} tokens, {shape.layers} layers",
            "ms_per_forward": round(statistics.median(times), 2),
            "per_op_ms": {k: round(v, 2) for k, v in per_op.items()}}


def package_load_case(args, torch, device) -> dict:
    """Start-up cost of a 7B-geometry runner (``--layers`` decoder layers):
    built from fp16 host weights (H2D of the fp16 bytes + per-output
    quantisation on the GPU, what a start without an int8 cache does) against
    built from the checksummed int8 package (read + SHA-256 of every file on
    the host thread pool + H2D of the int8 bytes). The package is written to
    a temporary directory first, so its files are in the page cache: the
    figure excludes the storage read."""
    import tempfile
    from dataclasses import replace
    from nanopointllm_b200 import package as P, runner as R, synthetic as S
    shape = replace(S.LLAMA_7B, layers=args.layers)
    lazy = S.LazyLlamaWeights(shape, seed=0, device=str(device))
    host = {name: lazy[name].cpu() for name in lazy.keys()}
    fp16_bytes = sum(t.numel() * 2 for t in host.values())

    def build(fn):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run = fn()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        del run
        torch.cuda.empty_cache()
        return dt

    with tempfile.TemporaryDirectory(prefix="npl_pkg_") as d:
        t0 = time.perf_counter()
        manifest = P.write_w8a8_llama_package(d, shape, host, device=device)
        t_write = time.perf_counter() - t0
        pkg_bytes = sum(int(e["bytes"]) for e in manifest["tensors"].values())
        t_float, t_pkg = [], []
        for _ in range(max(1, args.steps)):
            t_float.append(build(lambda: R.W8A8LlamaRunner(shape, host, device=device, num_blocks=1, block_size=256)))
            t_pkg.append(build(lambda: R.W8A8LlamaRunner.from_package(d, device=device, num_blocks=1,
                                                                      block_size=256)))
    tf, tp = statistics.median(t_float), statistics.median(t_pkg)
    return {"layers": shape.layers, "package_gb": round(pkg_bytes / 1e9, 3), "fp16_gb": round(fp16_bytes / 1e9, 3),
            "write_s": round(t_write, 2), "build_from_fp16_s": round(tf, 3), "build_from_package_s": round(tp, 3),
            "package_gbs": round(pkg_bytes / tp / 1e9, 2), "speedup": round(tf / tp, 2),
            "host_threads": os.cpu_count(), "note": "package files in the page cache (written just before)"}


def run_serve(args, torch, rank: int, world: int, device) -> dict | None:
    """Config 5: 256 requests (513 point-embedding rows + U{47..511} text
    tokens, outputs U{16, 64, 256}, all at t = 0) routed over the replicas
    (one per GPU, data parallel), each served by continuous batching
    (nanopointllm_b200.serving); output tokens/s of the whole job over the
    slowest replica's time."""
    from nanopointllm_b200 import runner as R, serving as SV, synthetic as S
    shape = S.LLAMA_7B if args.layers == 32 else S.LlamaShape(**{**S.LLAMA_7B.as_dict(), "layers": args.layers})
    from nanopointllm_b200 import tp as TP
    reqs = SV.config5_requests(args.serve_requests, vocab=shape.vocab)
    tp = args.tp and world > 1
    # data parallel: each replica serves its routed share with its own
    # weights; tensor parallel: every rank serves all requests in lock step
    share = reqs if tp else SV.route(reqs, world)[rank]
    max_len = max(q.n_point_rows + len(q.text_ids) + q.max_tokens for q in reqs)
    max_blocks = -(-max_len // BLOCK_SIZE)
    num_blocks = args.serve_max_seqs * max_blocks + 8
    cls = TP.W8A8TPLlamaRunner if tp else R.W8A8LlamaRunner
    kw = {"peer_exchange": not args.tp_nccl} if tp else {}
    run = cls(shape, S.LazyLlamaWeights(shape, seed=0 if tp else rank_seed(rank), device=str(device)),
              device=device, num_blocks=num_blocks, block_size=BLOCK_SIZE, **kw)
    eng = SV.ServingEngine(run, max_num_seqs=args.serve_max_seqs, max_num_batched_tokens=16384,
                           max_blocks_per_seq=max_blocks)
    res = eng.run(share)
    out = SV.gather_metrics(res) if world > 1 and not tp else SV.gather_metrics_local(res)
    eng.graphs.clear()  # releases the decode graphs (and any NCCL calls in them) before the process group goes
    torch.cuda.synchronize()
    if rank != 0:
        return None
    return {"metric": "config5 serving output tokens/s (continuous batching, greedy)",
            "value": round(out["output_tokens_per_s"], 1), "unit": "tokens/s", "n_gpus": world,
            "higher_is_better": True, "scaling": "strong", "dtype": "int8 (W8A8), fp16 attention",
            "data": "synthetic", "config": {"workload": f"config5: {len(reqs)} requests, 513 point rows + "
                                                        "U{47..511} text tokens, outputs U{16,64,256}",
                                            "parallelism": f"tp{world}" if tp else f"dp{world}",
                                            "max_num_seqs": args.serve_max_seqs,
                                            "block_size": BLOCK_SIZE},
            "serving": {k: (round(v, 4) if isinstance(v, float) else v) for k, v in out.items()},
            "steps": res["steps"], "step_wall_s": res["step_s"]}


def run_reference(args, rank: int, world: int) -> dict | None:
    """The reference arm: the reference's CPU W8A8 decode path on this box's
    host cores (rank 0 alone; with torchrun the other ranks leave first, so
    the timing runs with the host to itself). A bench step is one decoder
    layer of the 32 (they all cost the same): ``--warmup`` untimed layers,
    ``--steps`` timed ones, then the LM head; ``value`` is the full step's
    tokens/s, batch / (32 x mean layer + LM head)."""
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return None
        time.sleep(3.0)  # the other ranks' processes exit
    times, head, threads = cpu_layers(args.steps, args.warmup)
    step_s = cpu_step_seconds(times, head)
    v = round(BATCH / step_s, 4)
    cb = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
          "sample": f"per bench step one decoder layer (7B widths, batch 8, ctx 1024, paged KV) on the host CPU, "
                    f"{len(times)} timed after {args.warmup} warm-up, + the LM head once: torch int32 matmuls as "
                    f"integer_linear_per_output_reference, SDPA attention; full step = 32 x mean layer "
                    f"({statistics.mean(times):.3f} s) + head ({head:.3f} s)",
          "s_per_step": round(step_s, 3)}
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * statistics.mean(times), 1),
            "step": "one of the 32 decoder layers (ms_per_step is its measured mean time; value scales it to "
                    "the full 32-layer step + LM head)",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "impl": "reference",
            "dtype": "int8 (W8A8: int8 x int8 -> int32 on the CPU)", "data": "synthetic",
            "config": {"workload": "config3: W8A8 Llama-7B-arch decode step, batch 8, ctx 1024, block_size 256 "
                                   "(reference CPU path, rank 0 only)", "batch_per_gpu": BATCH, "context": CTX,
                       "layers": 32},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=32, help="fewer layers only for quick checks (not the metric)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--kernel-case", choices=KERNEL_CASES, help="run one op alone (profiling harness)")
    ap.add_argument("--serve", action="store_true", help="config 5 serving run instead of the decode metric")
    ap.add_argument("--tp", action="store_true",
                    help="tensor parallel over the N ranks (decode step, or --serve) instead of N replicas")
    ap.add_argument("--tp-nccl", action="store_true",
                    help="with --tp: NCCL all-reduces instead of the NVLink peer-memory exchanges")
    ap.add_argument("--serve-requests", type=int, default=256)
    ap.add_argument("--serve-max-seqs", type=int, default=64)
    ap.add_argument("--prefill-seqs", type=int, default=8, help="prefill_attention case: sequences")
    ap.add_argument("--prefill-len", type=int, default=560, help="prefill_attention case: tokens per sequence")
    ap.add_argument("--attn-batch", type=int, default=0, help="attention case: sequences (default 8)")
    ap.add_argument("--attn-ctx", type=int, nargs=2, metavar=("LO", "HI"),
                    help="attention case: contexts drawn uniformly from [LO, HI] (default 1040)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line:
            print(json.dumps(line))
        return 0

    import torch
    _register_package()
    dist = None
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.kernel_case:
        print(json.dumps(run_kernel_case(args, torch, device)))
        return 0
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    try:
        if args.serve:
            line = run_serve(args, torch, rank, world, device)
        elif args.tp:
            line = run_tp(args, torch, dist, rank, world, device)
        else:
            line = run_ours(args, torch, dist, rank, world, device)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    if line:
        print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
