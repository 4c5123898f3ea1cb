"""W8A8 Llama runner over the paged KV pool: the drop-in for the reference's
``LightweightLlamaRunner`` on the W8A8 path.

Reference structure followed (nanopointllm):
  engine/forward_context.py:10-39       ForwardContext (slot_mapping, block_tables,
                                          context_lens, position_ids, seq_lens)
  llama/lightweight_runner.py:625-736   LightweightLlamaRunner.forward
  llama/lightweight_runner.py:480-560   LightweightLlamaLayer.forward (eager semantics:
                                          RMSNorm, attention, fp16 residual, RMSNorm, MLP,
                                          fp16 residual)
  llama/paged_attention.py:1271-1488    PagedLlamaAttention.forward (QKV, rotary_fn,
                                          store_kvcache, decode / prefill attention, o_proj)
  engine/cuda_graph.py:30-77            strict decode CUDA-graph capture / replay
  engine/paged_model_runner.py:332-383  decode step: metadata in, greedy token out

Every Linear (packed QKV, O, packed gate/up, down, LM head) is W8A8: int8
weights quantised once per output channel, int8 activations quantised per
token, int32 accumulation on the tensor cores. A decode step runs nine
kernels of libnpl_w8a8 per layer and nothing else:

  RMSNorm+quant -> QKV -> RoPE + KV store -> paged attention [+quant] ->
  O [+residual] -> RMSNorm+quant -> gate/up [SiLU*up] -> quant ->
  down [+residual]

(brackets: fused into that kernel). Every kernel launches with programmatic
dependent launch, so the small normalisation / quantisation / RoPE kernels
overlap the launch and weight prefetch of the next linear. (Folding them into
the linears themselves -- the fp16-activation and RoPE modes of
npl_w8a8_linear_ex -- measured slower on B200: it lengthens the linear's
critical path by more than the small kernel costs.)

Prefill attention over multi-token rows is npl_paged_prefill_attention (the
tcgen05 replacement of the reference's Triton varlen kernel); the prefill
linears are the same tcgen05 kernels at M = prefill tokens.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F

from . import _lib as L
from . import package as P
from . import paged_attention as PA
from . import w8a8 as W
from .rope import rope_tables
from .synthetic import LlamaShape


# ------------------------------------------------------------------ context
@dataclass
class ForwardContext:
    """Per-step metadata, as nanopointllm/engine/forward_context.py:10-24."""
    slot_mapping: torch.Tensor                    # [T] int32, -1 = skip
    block_tables: Optional[torch.Tensor]          # [B, max_blocks] int32
    context_lens: Optional[torch.Tensor]          # [B] int32
    position_ids: Optional[torch.Tensor] = None   # [1, T] int64
    seq_lens: list[int] = field(default_factory=list)


_ctx = threading.local()


def set_forward_context(ctx: Optional[ForwardContext]) -> None:
    _ctx.value = ctx


def get_forward_context() -> Optional[ForwardContext]:
    return getattr(_ctx, "value", None)


def clear_forward_context() -> None:
    _ctx.value = None


# ------------------------------------------------------------ fused norm
def rmsnorm_quant(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None, *,
                  sum_out: torch.Tensor | None = None, normed_out: torch.Tensor | None = None):
    """RMSNorm (of x + residual when given) fused with per-token int8
    quantisation. Returns (q int8 [M, K], scale fp32 [M], sum_out)."""
    m, k = x.shape
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    if residual is not None and sum_out is None:
        sum_out = torch.empty_like(x)
    L.check(L.lib.npl_rmsnorm_quant(x.data_ptr(), L.ptr(residual), weight.data_ptr(), float(eps), m, k,
                                    L.ptr(sum_out), L.ptr(normed_out), q.data_ptr(), s.data_ptr(),
                                    L.stream_ptr(x.device)))
    return q, s, sum_out


def shape_from_hf_config(cfg) -> LlamaShape:
    """LlamaShape of an HF LlamaConfig (transformers 4.x rope_theta or 5.x
    rope_parameters; head_dim defaults to hidden / heads)."""
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    rope = getattr(cfg, "rope_parameters", None) or {}
    theta = rope.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))
    kv_heads = getattr(cfg, "num_key_value_heads", None) or cfg.num_attention_heads
    return LlamaShape(hidden=cfg.hidden_size, heads=cfg.num_attention_heads, kv_heads=kv_heads,
                      head_dim=head_dim, intermediate=cfg.intermediate_size, layers=cfg.num_hidden_layers,
                      vocab=cfg.vocab_size, rope_theta=float(theta), eps=cfg.rms_norm_eps,
                      max_position=cfg.max_position_embeddings)


class W8A8Layer:
    def __init__(self, shape: LlamaShape, src, idx: int, device: torch.device,
                 k_cache: torch.Tensor, v_cache: torch.Tensor):
        """``src``: a weight source (package.FloatLlamaWeights or
        package.PackagedLlamaWeights) giving each Linear's int8 weight and
        per-output scales and the fp16 norm weights."""
        p = f"model.layers.{idx}."
        qkv = [src.linear(p + "self_attn." + n) for n in ("q_proj", "k_proj", "v_proj")]
        self.qkv = W.W8A8Linear(torch.cat([q for q, _ in qkv]), torch.cat([s for _, s in qkv]))
        self.o = W.W8A8Linear(*src.linear(p + "self_attn.o_proj"))
        gq, gs = src.linear(p + "mlp.gate_proj")
        uq, us = src.linear(p + "mlp.up_proj")
        self.gate_up = W.W8A8Linear(W.pack_gate_up(gq, uq), W.pack_gate_up(gs, us))
        self.down = W.W8A8Linear(*src.linear(p + "mlp.down_proj"))
        self.input_norm = src.dense(p + "input_layernorm.weight")
        self.post_norm = src.dense(p + "post_attention_layernorm.weight")
        self.k_cache = k_cache
        self.v_cache = v_cache


class W8A8LlamaRunner:
    """Replaces LightweightLlamaRunner for W8A8 serving on sm_100a.

    ``forward(input_ids | inputs_embeds, position_ids)`` reads the paged
    metadata from the thread-local ForwardContext and returns fp16 logits
    [1, T, vocab] (or only each sequence's last row with ``last_only=True``).

    ``state_dict``: HF-named float weights (each Linear is quantised per
    output channel on the GPU as its layer is built) or a weight source with
    linear()/dense(), e.g. a checksummed int8 package (see from_package).
    """

    def __init__(self, shape: LlamaShape, state_dict: dict[str, torch.Tensor], *, device: torch.device,
                 kv_pool: torch.Tensor | None = None, num_blocks: int = 0, block_size: int = 256,
                 fuse_mlp_quant: bool = False, fuse_silu_quant: bool = False, forward_context=None):
        """``forward_context``: a callable returning the current step's
        context. Default: this module's get_forward_context. The reference
        engine passes its own nanopointllm.engine.forward_context.
        get_forward_context; its ForwardContext (forward_context.py:10-24) is
        read as it is, through the fields slot_mapping, block_tables,
        context_lens, position_ids and seq_lens."""
        self.shape = shape
        self.device = torch.device(device)
        self.forward_context = forward_context or get_forward_context
        # fuse_mlp_quant, decode batches (<= 64 tokens): the gate/up epilogue
        # also records each token's absmax of SiLU(gate)*up, and down quantises
        # its fp16 input itself, so no separate quantisation kernel runs between
        # them. Off by default: on B200 the in-kernel quantisation lengthens
        # down's critical path by more than the separate kernel costs.
        self.fuse_mlp_quant = fuse_mlp_quant
        # fuse_silu_quant, decode batches: the gate/up launch also quantises
        # SiLU(gate)*up per token once all of its CTAs have stored their
        # outputs (a grid-wide count), so down takes int8 rows with no
        # quantisation launch between them; bit-identical to the separate
        # kernel. Off by default: on B200 the grid-wide wait and the extra
        # pass lengthen gate/up by as much as the separate launch costs
        # (decode step 3.289 ms against 3.279).
        self.fuse_silu_quant = fuse_silu_quant
        self._act_absmax = torch.zeros(64, dtype=torch.int32, device=self.device)
        if kv_pool is None:
            kv_pool = torch.zeros(2, shape.layers, num_blocks, block_size, shape.kv_heads, shape.head_dim,
                                  dtype=torch.float16, device=self.device)
        if kv_pool.dim() != 6 or kv_pool.dtype != torch.float16:
            raise ValueError("kv_pool must be fp16 [2, layers, num_blocks, block_size, Hkv, D]")
        self.kv_pool = kv_pool
        self.block_size = kv_pool.shape[3]
        self.num_blocks = kv_pool.shape[2]
        src = P.as_weight_source(state_dict, self.device)
        self.embed = src.dense("model.embed_tokens.weight")
        self.layers = [W8A8Layer(shape, src, i, self.device, kv_pool[0, i], kv_pool[1, i])
                       for i in range(shape.layers)]
        self.norm = src.dense("model.norm.weight")
        self.lm_head = W.W8A8Linear(*src.linear("lm_head"))
        self.cos, self.sin = rope_tables(shape.head_dim, shape.max_position, shape.rope_theta, self.device)
        self.scale = shape.head_dim ** -0.5

    @classmethod
    def from_package(cls, directory, *, device: torch.device, **kwargs):
        """Builds the runner from a whole-model int8 package
        (package.write_w8a8_llama_package) instead of float weights: no
        weight is re-quantised, and every tensor is SHA-256-checked before it
        reaches the GPU. kwargs as the constructor's (kv_pool, num_blocks,
        block_size, ...)."""
        src = P.PackagedLlamaWeights(directory, device)
        try:
            return cls(src.shape, src, device=device, **kwargs)
        finally:
            src.close()

    @classmethod
    def from_hf(cls, hf_model, kv_pool: torch.Tensor, device: torch.device | None = None,
                forward_context=None) -> "W8A8LlamaRunner":
        """Build from an HF LlamaForCausalLM (the engine's model) and the
        engine's KV pool tensor (KVPool.pool, kv_pool.py:9-24); every Linear
        of the model is quantised per output channel once, here.
        ``forward_context`` as the constructor's."""
        shape = shape_from_hf_config(hf_model.config)
        device = device or kv_pool.device
        return cls(shape, dict(hf_model.state_dict()), device=device, kv_pool=kv_pool,
                   forward_context=forward_context)

    # ------------------------------------------------------------- layers
    def _attention_q(self, layer: W8A8Layer, q: torch.Tensor, ctx: ForwardContext):
        """q [T, H, D] (rotated) -> per-token int8 attention rows [T, H*D] +
        fp32 scales [T] (the O projection's input). In decode steps the
        quantisation is fused into the attention kernel."""
        s = self.shape
        t = q.shape[0]
        if all(n == 1 for n in ctx.seq_lens):
            q8 = torch.empty((t, s.heads * s.head_dim), dtype=torch.int8, device=q.device)
            qs = torch.empty((t,), dtype=torch.float32, device=q.device)
            PA.paged_decode_attention(q, layer.k_cache, layer.v_cache, ctx.block_tables, ctx.context_lens,
                                      self.scale, s.heads // s.kv_heads, quant_out=(q8, qs))
            return q8, qs
        q8, qs = W.dynamic_per_token_quant(self._attention(layer, q, ctx))
        return q8, qs.reshape(-1)

    def _attention(self, layer: W8A8Layer, q: torch.Tensor, ctx: ForwardContext) -> torch.Tensor:
        """q [T, H, D] (rotated) -> [T, H*D] fp16."""
        s = self.shape
        t = q.shape[0]
        if all(n == 1 for n in ctx.seq_lens):
            out = PA.paged_decode_attention(q, layer.k_cache, layer.v_cache, ctx.block_tables, ctx.context_lens,
                                            self.scale, s.heads // s.kv_heads)
            return out.reshape(t, -1)
        # mixed / prefill step (paged_attention.py:1379-1440): the multi-token
        # rows of every sequence in one launch of the varlen prefill kernel,
        # single-token rows through the decode kernel
        groups = s.heads // s.kv_heads
        out = torch.empty((t, s.heads, s.head_dim), dtype=torch.float16, device=q.device)
        offs = [0]
        for n in ctx.seq_lens:
            offs.append(offs[-1] + n)
        pre = [i for i, n in enumerate(ctx.seq_lens) if n > 1]
        dec = [i for i, n in enumerate(ctx.seq_lens) if n == 1]
        dev = q.device
        if pre:
            rows = torch.tensor(pre, dtype=torch.long, device=dev)
            PA.paged_varlen_attention(
                q, layer.k_cache, layer.v_cache, ctx.block_tables.index_select(0, rows),
                ctx.context_lens.index_select(0, rows),
                torch.tensor([ctx.seq_lens[i] for i in pre], dtype=torch.int32, device=dev),
                torch.tensor([offs[i] for i in pre], dtype=torch.int32, device=dev), self.scale, groups,
                max_q_len=max(ctx.seq_lens[i] for i in pre), out=out)
        if dec:
            rows = torch.tensor(dec, dtype=torch.long, device=dev)
            at = torch.tensor([offs[i] for i in dec], dtype=torch.long, device=dev)
            o = PA.paged_decode_attention(q.index_select(0, at), layer.k_cache, layer.v_cache,
                                          ctx.block_tables.index_select(0, rows), ctx.context_lens.index_select(0, rows),
                                          self.scale, groups)
            out.index_copy_(0, at, o)
        return out.reshape(t, -1)

    # Optional per-op timing hook: timer(name, fn, *args, **kwargs) -> fn(...)
    # (used by bench.py to time each kernel with CUDA events on its stream).
    timer = None

    def _op(self, name: str, fn, *args, **kwargs):
        if self.timer is None:
            return fn(*args, **kwargs)
        return self.timer(name, fn, *args, **kwargs)

    def _layer(self, layer: W8A8Layer, h: torch.Tensor, positions: torch.Tensor, ctx: ForwardContext):
        s, op = self.shape, self._op
        xq, xs, _ = op("rmsnorm_quant", rmsnorm_quant, h, layer.input_norm, s.eps)
        qkv = op("linear.qkv", W.linear_q, xq, xs, layer.qkv.qweight, layer.qkv.wscale)
        q = op("rope_store", PA.rope_store_kvcache, qkv, s.heads, s.kv_heads, s.head_dim, self.cos, self.sin,
               positions, ctx.slot_mapping, layer.k_cache, layer.v_cache)
        aq, asc = op("attention", self._attention_q, layer, q, ctx)
        h2 = op("linear.o", W.linear_q, aq, asc, layer.o.qweight, layer.o.wscale,
                epilogue=L.EPI_RESIDUAL, residual=h)
        xq, xs, _ = op("rmsnorm_quant", rmsnorm_quant, h2, layer.post_norm, s.eps)
        m = h2.shape[0]
        if self.fuse_mlp_quant and m <= self._act_absmax.numel():
            # the absmax buffer is zero on entry and zeroed again by down
            act = op("linear.gate_up", W.linear_ex, layer.gate_up.qweight, layer.gate_up.wscale, x_mode=L.X_INT8,
                     m=m, qa=xq, sa=xs, epilogue=L.EPI_SILU_MUL, absmax_out=self._act_absmax)
            return op("linear.down", W.linear_ex, layer.down.qweight, layer.down.wscale, x_mode=L.X_F16_ABSMAX,
                      m=m, x_f16=act, x_absmax=self._act_absmax, epilogue=L.EPI_RESIDUAL, residual=h2)
        if self.fuse_silu_quant and m <= self._act_absmax.numel():
            inter = layer.gate_up.qweight.shape[0] // 2
            aq = torch.empty((m, inter), dtype=torch.int8, device=h2.device)
            asc = torch.empty(m, dtype=torch.float32, device=h2.device)
            # the absmax buffer is zero on entry and zeroed again by the launch
            op("linear.gate_up", W.linear_ex, layer.gate_up.qweight, layer.gate_up.wscale, x_mode=L.X_INT8, m=m,
               qa=xq, sa=xs, epilogue=L.EPI_SILU_MUL, absmax_out=self._act_absmax, q_out=aq, q_scale=asc)
            return op("linear.down", W.linear_q, aq, asc, layer.down.qweight, layer.down.wscale,
                      epilogue=L.EPI_RESIDUAL, residual=h2)
        act = op("linear.gate_up", W.linear_q, xq, xs, layer.gate_up.qweight, layer.gate_up.wscale,
                 epilogue=L.EPI_SILU_MUL)
        aq, asc = op("quant", W.dynamic_per_token_quant, act)
        return op("linear.down", W.linear_q, aq, asc.reshape(-1), layer.down.qweight, layer.down.wscale,
                  epilogue=L.EPI_RESIDUAL, residual=h2)

    @torch.inference_mode()
    def forward(self, input_ids: torch.Tensor | None = None, *, inputs_embeds: torch.Tensor | None = None,
                position_ids: torch.Tensor | None = None, last_only: bool = False) -> torch.Tensor:
        ctx = self.forward_context()
        if ctx is None:
            raise RuntimeError("W8A8LlamaRunner.forward needs a ForwardContext (set_forward_context)")
        if inputs_embeds is None:
            if input_ids is None:
                raise ValueError("input_ids or inputs_embeds is required")
            h = F.embedding(input_ids.reshape(-1), self.embed)
        else:
            h = inputs_embeds.reshape(-1, self.shape.hidden).to(torch.float16).contiguous()
        pos = position_ids if position_ids is not None else ctx.position_ids
        pos = pos.reshape(-1).to(torch.int64).contiguous()
        for layer in self.layers:
            h = self._layer(layer, h, pos, ctx)
        if last_only and not all(n == 1 for n in ctx.seq_lens):
            last = torch.tensor([sum(ctx.seq_lens[:i + 1]) - 1 for i in range(len(ctx.seq_lens))],
                                device=h.device)
            h = h.index_select(0, last).contiguous()
        xq, xs, _ = self._op("rmsnorm_quant", rmsnorm_quant, h, self.norm, self.shape.eps)
        return self._lm_head(xq, xs).unsqueeze(0)

    def _lm_head(self, xq: torch.Tensor, xs: torch.Tensor) -> torch.Tensor:
        """int8 final-norm rows [T, hidden] + scales -> fp16 logits [T, vocab]."""
        return self._op("linear.lm_head", W.linear_q, xq, xs, self.lm_head.qweight, self.lm_head.wscale)

    __call__ = forward


class DecodeGraph:
    """Strict CUDA-graph decode step for a fixed batch and block-table width
    (engine/cuda_graph.py:30-77): static metadata buffers, one replay per step,
    greedy argmax inside the graph."""

    def __init__(self, runner: W8A8LlamaRunner, batch: int, max_blocks: int):
        dev = runner.device
        self.runner = runner
        self.ids = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.slots = torch.full((batch,), -1, dtype=torch.int32, device=dev)
        self.context_lens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.block_tables = torch.zeros(batch, max_blocks, dtype=torch.int32, device=dev)
        self.ctx = ForwardContext(slot_mapping=self.slots, block_tables=self.block_tables,
                                  context_lens=self.context_lens, position_ids=self.positions,
                                  seq_lens=[1] * batch)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.logits: torch.Tensor | None = None
        self.next_tokens: torch.Tensor | None = None

    def _run(self):
        set_forward_context(self.ctx)
        try:
            logits = self.runner.forward(self.ids, position_ids=self.positions)
        finally:
            clear_forward_context()
        return logits, torch.argmax(logits[0], dim=-1)

    def capture(self) -> None:
        s = torch.cuda.Stream(device=self.runner.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # sizes every workspace before capture
                self._run()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.logits, self.next_tokens = self._run()
        self.graph = g

    def load(self, ids, positions, slots, context_lens, block_tables, non_blocking: bool = True) -> None:
        self.ids.copy_(ids, non_blocking=non_blocking)
        self.positions.copy_(positions, non_blocking=non_blocking)
        self.slots.copy_(slots, non_blocking=non_blocking)
        self.context_lens.copy_(context_lens, non_blocking=non_blocking)
        self.block_tables.copy_(block_tables, non_blocking=non_blocking)

    def replay(self) -> torch.Tensor:
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()
        return self.next_tokens
