"""Tensor-parallel W8A8 Llama runner: one process per GPU, torch.distributed
(NCCL) for the exchanges.

The split follows the tensor-parallel variant of the reference's serving
configuration (one exchange per row-parallel linear):

* column-parallel: the packed QKV projection (rank r owns q heads
  [r H/P, (r+1) H/P) and kv heads [r Hkv/P, ...), and the KV-pool slice of
  its kv heads), gate/up (rows [r I/P, ...) of gate and of up, each rank's
  slice zero-padded to a multiple of 64 rows for the interleaved
  SiLU*up epilogue) and the LM head (vocab rows; logits all-gathered);
* row-parallel: O and down. Their int8 input rows are split over the ranks,
  but the per-token scale is that of the WHOLE row (w8a8.py:106-115), so each
  rank takes the absmax of its part (npl_row_absmax), the ranks all-reduce it
  with MAX, and quantise with it (npl_quant_rows_absmax); each rank's linear
  then yields int32 partial accumulators over its K slice, the ranks
  all-reduce them with SUM (exact), and npl_dequant applies the dequant +
  residual epilogue.

Weights are quantised per output channel from the FULL weight before they are
sliced, so every per-row scale equals the single-GPU one; together with exact
int32 sums and the whole-row activation scales this makes the tensor-parallel
forward bit-identical to W8A8LlamaRunner's. RMSNorm, residuals and the
embedding are replicated.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import torch
import torch.distributed as dist

from . import _lib as L
from . import package as P
from . import paged_attention as PA
from . import w8a8 as W
from .rope import rope_tables
from . import runner as R
from .runner import ForwardContext, W8A8LlamaRunner, rmsnorm_quant
from .synthetic import LlamaShape

TILE_PAIR = 64  # gate/up rows per half tile of the SiLU*up epilogue


@dataclass(frozen=True)
class TPPlan:
    """Which slices of each weight rank `rank` of `world` owns."""
    rank: int
    world: int
    h0: int        # first q head
    hl: int        # q heads per rank
    kv0: int       # first kv head
    kvl: int       # kv heads per rank
    i0: int        # first intermediate row
    i1: int        # end of the intermediate rows (exclusive)
    il_pad: int    # intermediate rows per rank, padded to a multiple of 64
    v0: int        # first vocab row
    v1: int        # end of the vocab rows (exclusive)
    vl_pad: int    # vocab rows per rank (equal on every rank, for the all-gather)


def tp_plan(shape: LlamaShape, rank: int, world: int) -> TPPlan:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    if shape.heads % world or shape.kv_heads % world:
        raise ValueError(f"{shape.heads} q heads / {shape.kv_heads} kv heads do not split over {world} ranks")
    hl, kvl = shape.heads // world, shape.kv_heads // world
    il = -(-shape.intermediate // world)
    i0, i1 = min(rank * il, shape.intermediate), min((rank + 1) * il, shape.intermediate)
    il_pad = -(-il // TILE_PAIR) * TILE_PAIR
    vl = -(-shape.vocab // world)
    v0, v1 = min(rank * vl, shape.vocab), min((rank + 1) * vl, shape.vocab)
    return TPPlan(rank, world, rank * hl, hl, rank * kvl, kvl, i0, i1, il_pad, v0, v1, vl)


def qkv_rows(shape: LlamaShape, plan: TPPlan) -> torch.Tensor:
    """Row indices of the packed [q | k | v] projection this rank owns."""
    d, hq, hk = shape.head_dim, shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    q = torch.arange(plan.h0 * d, (plan.h0 + plan.hl) * d)
    k = torch.arange(plan.kv0 * d, (plan.kv0 + plan.kvl) * d) + hq
    v = torch.arange(plan.kv0 * d, (plan.kv0 + plan.kvl) * d) + hq + hk
    return torch.cat([q, k, v])


def pad_rows(t: torch.Tensor, rows: int, fill: float = 0.0) -> torch.Tensor:
    if t.shape[0] == rows:
        return t.contiguous()
    out = torch.full((rows, *t.shape[1:]), fill, dtype=t.dtype, device=t.device)
    out[:t.shape[0]] = t
    return out


def pad_cols(t: torch.Tensor, cols: int) -> torch.Tensor:
    out = torch.zeros((t.shape[0], cols), dtype=t.dtype, device=t.device)
    out[:, :t.shape[1]] = t
    return out


# per-row scale of an all-zero weight row (scale_from_absmax(0) = fp16.tiny)
ZERO_ROW_SCALE = 2.0 ** -14


class W8A8TPLayer:
    def __init__(self, shape: LlamaShape, plan: TPPlan, src, idx: int, device: torch.device,
                 k_cache: torch.Tensor, v_cache: torch.Tensor):
        """``src`` gives the FULL int8 weights and per-row scales (quantised
        from float weights, or read from a package); this rank keeps its
        slices."""
        p = f"model.layers.{idx}."
        qkv = [src.linear(p + "self_attn." + n) for n in ("q_proj", "k_proj", "v_proj")]
        qkv_q, qkv_s = torch.cat([q for q, _ in qkv]), torch.cat([s for _, s in qkv])
        rows = qkv_rows(shape, plan).to(device)
        self.qkv = W.W8A8Linear(qkv_q[rows], qkv_s[rows])
        d = shape.head_dim
        oq, os_ = src.linear(p + "self_attn.o_proj")
        self.o = W.W8A8Linear(oq[:, plan.h0 * d:(plan.h0 + plan.hl) * d], os_)
        gq, gs = src.linear(p + "mlp.gate_proj")
        uq, us = src.linear(p + "mlp.up_proj")
        sl = slice(plan.i0, plan.i1)
        self.gate_up = W.W8A8Linear(
            W.pack_gate_up(pad_rows(gq[sl], plan.il_pad), pad_rows(uq[sl], plan.il_pad)),
            W.pack_gate_up(pad_rows(gs[sl], plan.il_pad, ZERO_ROW_SCALE), pad_rows(us[sl], plan.il_pad, ZERO_ROW_SCALE)))
        dq, ds = src.linear(p + "mlp.down_proj")
        self.down = W.W8A8Linear(pad_cols(dq[:, sl], plan.il_pad), ds)
        self.input_norm = src.dense(p + "input_layernorm.weight")
        self.post_norm = src.dense(p + "post_attention_layernorm.weight")
        self.k_cache = k_cache
        self.v_cache = v_cache


class PeerExchange:
    """The NVLink peer-memory exchanges of the row-parallel linears for decode
    batches (<= 64 tokens): one zero-filled exchange buffer per rank, mapped by
    every other rank through CUDA IPC (npl_ipc_*). ``absmax_quant`` and
    ``allreduce_dequant`` give exactly what the NCCL path gives
    (row_absmax + all-reduce(MAX) + quant_rows_absmax, and all-reduce(SUM) +
    dequant) in one kernel each. Every rank must make the same calls in the
    same order."""

    MAX_ROWS = 64

    def __init__(self, group: dist.ProcessGroup, device: torch.device, max_cols: int):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > L.TP_MAX_RANKS:
            raise ValueError(f"at most {L.TP_MAX_RANKS} ranks")
        self.max_elems = self.MAX_ROWS * (-(-max_cols // 4) * 4)
        nbytes = int(L.lib.npl_tp_exchange_bytes(self.world, self.max_elems))
        # 256-byte aligned start: the allocator returns 512-byte aligned blocks
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        handle = ctypes.create_string_buffer(L.IPC_HANDLE_BYTES)
        offset = ctypes.c_size_t(0)
        with torch.cuda.device(device):
            L.check(L.lib.npl_ipc_handle(self.buf.data_ptr(), handle, ctypes.byref(offset)))
        torch.cuda.synchronize(device)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, (handle.raw, offset.value), group=group)
        self._opened: list[int] = []
        ptrs = []
        with torch.cuda.device(device):
            for r, (h, off) in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.buf.data_ptr())
                    continue
                p_out, b_out = ctypes.c_void_p(), ctypes.c_void_p()
                L.check(L.lib.npl_ipc_open(h, off, ctypes.byref(p_out), ctypes.byref(b_out)))
                self._opened.append(b_out.value)
                ptrs.append(p_out.value)
        self.peers = L.NplTpPeers(self.world, self.rank, (ctypes.c_void_p * L.TP_MAX_RANKS)(*ptrs),
                                  self.max_elems)
        dist.barrier(group=group)  # every buffer is zero and mapped before the first push

    def usable(self, m: int, n: int) -> bool:
        return 0 < m <= self.MAX_ROWS and m * n <= self.max_elems and n % 4 == 0

    def absmax_quant(self, x16: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        m, k = x16.shape
        q = torch.empty((m, k), dtype=torch.int8, device=x16.device)
        s = torch.empty((m,), dtype=torch.float32, device=x16.device)
        L.check(L.lib.npl_tp_absmax_quant(ctypes.byref(self.peers), x16.data_ptr(), m, k, x16.stride(0),
                                          q.data_ptr(), q.stride(0), s.data_ptr(), L.stream_ptr(x16.device)))
        return q, s

    def allreduce_dequant(self, acc: torch.Tensor, sa: torch.Tensor, wscale: torch.Tensor,
                          residual: torch.Tensor | None) -> torch.Tensor:
        m, n = acc.shape
        out = torch.empty((m, n), dtype=torch.float16, device=acc.device)
        L.check(L.lib.npl_tp_allreduce_dequant(
            ctypes.byref(self.peers), acc.data_ptr(), m, n, sa.data_ptr(), wscale.data_ptr(), None,
            L.ptr(residual), 0 if residual is None else residual.stride(0), out.data_ptr(), out.stride(0),
            L.stream_ptr(acc.device)))
        return out

    def close(self) -> None:
        for b in self._opened:
            L.lib.npl_ipc_close(b)
        self._opened = []


class W8A8TPLlamaRunner(W8A8LlamaRunner):
    """W8A8LlamaRunner split over the ranks of `group` (one GPU each). The
    calling convention is the same (forward reads the ForwardContext and
    returns the full fp16 logits [1, T, vocab] on every rank); the KV pool
    holds this rank's kv heads: [2, layers, num_blocks, block_size, Hkv / P, D]."""

    def __init__(self, shape: LlamaShape, state_dict: dict[str, torch.Tensor], *, device: torch.device,
                 group: dist.ProcessGroup | None = None, num_blocks: int = 0, block_size: int = 256,
                 kv_pool: torch.Tensor | None = None, peer_exchange: bool = True, forward_context=None):
        """``peer_exchange``: decode batches (<= 64 tokens) exchange the
        row-parallel absmax and int32 partials through NVLink peer memory
        (PeerExchange) instead of NCCL all-reduces; larger batches use NCCL.
        Results are identical either way. ``forward_context`` as
        W8A8LlamaRunner's."""
        self.group = group if group is not None else dist.group.WORLD
        self.plan = tp_plan(shape, dist.get_rank(self.group), dist.get_world_size(self.group))
        self.full_shape = shape
        # the local geometry the attention path sees
        self.shape = replace(shape, heads=self.plan.hl, kv_heads=self.plan.kvl)
        self.device = torch.device(device)
        self.forward_context = forward_context or R.get_forward_context
        self.fuse_mlp_quant = False
        self.timer = None
        if kv_pool is None:
            kv_pool = torch.zeros(2, shape.layers, num_blocks, block_size, self.plan.kvl, shape.head_dim,
                                  dtype=torch.float16, device=self.device)
        if kv_pool.dim() != 6 or kv_pool.shape[4] != self.plan.kvl:
            raise ValueError("kv_pool must be fp16 [2, layers, num_blocks, block_size, Hkv / world, D]")
        self.kv_pool = kv_pool
        self.block_size = kv_pool.shape[3]
        self.num_blocks = kv_pool.shape[2]
        src = P.as_weight_source(state_dict, self.device)
        self.embed = src.dense("model.embed_tokens.weight")
        self.layers = [W8A8TPLayer(shape, self.plan, src, i, self.device, kv_pool[0, i], kv_pool[1, i])
                       for i in range(shape.layers)]
        self.norm = src.dense("model.norm.weight")
        hq, hs = src.linear("lm_head")
        vs = slice(self.plan.v0, self.plan.v1)
        self.lm_head = W.W8A8Linear(pad_rows(hq[vs], self.plan.vl_pad), pad_rows(hs[vs], self.plan.vl_pad,
                                                                                 ZERO_ROW_SCALE))
        self.cos, self.sin = rope_tables(shape.head_dim, shape.max_position, shape.rope_theta, self.device)
        self.scale = shape.head_dim ** -0.5
        self.xchg = PeerExchange(self.group, self.device, shape.hidden) \
            if peer_exchange and self.plan.world > 1 else None

    # --------------------------------------------------------- exchanges
    def _allreduce(self, t: torch.Tensor, op) -> torch.Tensor:
        dist.all_reduce(t, op=op, group=self.group)
        return t

    def _row_parallel(self, x16: torch.Tensor, lin: W.W8A8Linear, residual: torch.Tensor) -> torch.Tensor:
        """fp16 rows [T, K/P] (this rank's part of each row) -> fp16
        residual + x @ W^T over the whole K."""
        x = self.xchg
        if x is not None and x.usable(x16.shape[0], lin.out_features):
            xq, xs = x.absmax_quant(x16)
            acc = torch.empty((x16.shape[0], lin.out_features), dtype=torch.int32, device=x16.device)
            scratch = torch.empty((x16.shape[0], lin.out_features), dtype=torch.float16, device=x16.device)
            W.linear_q(xq, xs, lin.qweight, lin.wscale, out=scratch, acc_out=acc)
            return x.allreduce_dequant(acc, xs, lin.wscale, residual)
        amax = self._allreduce(W.row_absmax(x16), dist.ReduceOp.MAX)  # whole-row absmax (fp32 bits)
        xq, xs = W.quant_rows_absmax(x16, amax)
        acc = torch.empty((x16.shape[0], lin.out_features), dtype=torch.int32, device=x16.device)
        scratch = torch.empty((x16.shape[0], lin.out_features), dtype=torch.float16, device=x16.device)
        W.linear_q(xq, xs, lin.qweight, lin.wscale, out=scratch, acc_out=acc)
        self._allreduce(acc, dist.ReduceOp.SUM)  # int32 partial sums: exact
        return W.dequant(acc, xs, lin.wscale, residual=residual)

    def _layer(self, layer: W8A8TPLayer, h: torch.Tensor, positions: torch.Tensor, ctx: ForwardContext):
        s, op = self.shape, self._op
        xq, xs, _ = op("rmsnorm_quant", rmsnorm_quant, h, layer.input_norm, s.eps)
        qkv = op("linear.qkv", W.linear_q, xq, xs, layer.qkv.qweight, layer.qkv.wscale)
        q = op("rope_store", PA.rope_store_kvcache, qkv, s.heads, s.kv_heads, s.head_dim, self.cos, self.sin,
               positions, ctx.slot_mapping, layer.k_cache, layer.v_cache)
        attn = op("attention", self._attention, layer, q, ctx)
        h2 = op("linear.o", self._row_parallel, attn, layer.o, h)
        xq, xs, _ = op("rmsnorm_quant", rmsnorm_quant, h2, layer.post_norm, s.eps)
        act = op("linear.gate_up", W.linear_q, xq, xs, layer.gate_up.qweight, layer.gate_up.wscale,
                 epilogue=L.EPI_SILU_MUL)
        return op("linear.down", self._row_parallel, act, layer.down, h2)

    def _lm_head(self, xq: torch.Tensor, xs: torch.Tensor) -> torch.Tensor:
        local = self._op("linear.lm_head", W.linear_q, xq, xs, self.lm_head.qweight, self.lm_head.wscale)
        t = local.shape[0]
        gathered = torch.empty((self.plan.world, t, self.plan.vl_pad), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(gathered, local.contiguous(), group=self.group)
        return gathered.permute(1, 0, 2).reshape(t, -1)[:, :self.full_shape.vocab]
