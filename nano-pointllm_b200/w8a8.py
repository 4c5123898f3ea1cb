"""The W8A8 contract on the GPU, mirroring ``nanopointllm.compression.w8a8``.

Same numerics as the reference (w8a8.py:14-139): symmetric int8 in
[-127, 127], round-to-nearest-even, fp16-stored scales held as fp32,
int8 x int8 -> int32 accumulation, dequant ((acc * s_a) * s_w) + bias in fp32.
Every function runs the CUDA kernels of libnpl_w8a8 through its C ABI; inputs
must be CUDA tensors (there is no CPU path).
"""
from __future__ import annotations

import ctypes
from dataclasses import asdict, dataclass
from typing import Any

import torch

from . import _lib as L


@dataclass(frozen=True)
class W8A8Contract:
    """w8a8.py:14-30, unchanged."""
    weight_bits: int = 8
    activation_bits: int = 8
    symmetric_min: int = -127
    symmetric_max: int = 127
    rounding: str = "round_to_nearest_ties_to_even"
    scale_storage: str = "float16"
    accumulator: str = "signed_int32"
    bias: str = "floating_point_after_dequantization"
    nonlinear_norm_residual: str = "bf16_or_fp16"

    def as_dict(self) -> dict[str, Any]:
        return asdict(self)


CONTRACT = W8A8Contract()

_DT = {torch.float32: L.NPL_F32, torch.float16: L.NPL_F16}


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("the W8A8 path runs on CUDA tensors only")


def _rows(t: torch.Tensor) -> torch.Tensor:
    t = t.reshape(-1, t.shape[-1])
    return t if t.stride(-1) == 1 and t.stride(0) % 16 == 0 else t.contiguous()


def dynamic_per_token_quant(values: torch.Tensor, *, out: torch.Tensor | None = None,
                            scale_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """w8a8.py:106-115 (quantise step of dynamic_per_token_activation_qdq).

    Returns (q int8 [..., K], scales fp32 [..., 1]).
    """
    _require_cuda(values)
    if values.dtype not in _DT:
        raise ValueError("values must be float16 or float32")
    x = _rows(values)
    rows, k = x.shape
    q = out if out is not None else torch.empty((rows, k), dtype=torch.int8, device=x.device)
    s = scale_out if scale_out is not None else torch.empty((rows,), dtype=torch.float32, device=x.device)
    if rows == 0:  # nothing to launch (an empty tensor may have no device address)
        return q.reshape(values.shape), s.reshape(*values.shape[:-1], 1)
    L.check(L.lib.npl_quant_rows(x.data_ptr(), _DT[x.dtype], rows, k, x.stride(0), q.data_ptr(), q.stride(0),
                                 s.data_ptr(), L.stream_ptr(x.device)))
    return q.reshape(values.shape), s.reshape(*values.shape[:-1], 1)


def row_absmax(values: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row max |v| of [rows, K] (fp16/fp32) as fp32 bit patterns in int32
    [rows] (non-negative floats order like their bits, so a MAX all-reduce of
    these int32 values is the max of the floats)."""
    _require_cuda(values)
    x = _rows(values)
    rows, k = x.shape
    out = out if out is not None else torch.empty((rows,), dtype=torch.int32, device=x.device)
    L.check(L.lib.npl_row_absmax(x.data_ptr(), _DT[x.dtype], rows, k, x.stride(0), out.data_ptr(),
                                 L.stream_ptr(x.device)))
    return out


def quant_rows_absmax(values: torch.Tensor, absmax: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """dynamic_per_token_quant with the per-row absmax given (int32 fp32 bits,
    e.g. reduced over the ranks that each hold part of the row): (q int8
    [rows, K], scales fp32 [rows])."""
    _require_cuda(values, absmax)
    x = _rows(values)
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8, device=x.device)
    s = torch.empty((rows,), dtype=torch.float32, device=x.device)
    L.check(L.lib.npl_quant_rows_absmax(x.data_ptr(), _DT[x.dtype], rows, k, x.stride(0), absmax.data_ptr(),
                                        q.data_ptr(), q.stride(0), s.data_ptr(), L.stream_ptr(x.device)))
    return q, s


def dequant(acc: torch.Tensor, sa: torch.Tensor, wscale: torch.Tensor, *, bias: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """int32 accumulators [M, N] -> ((acc * sa) * sw) + bias (+ residual in
    fp16), as the linear's epilogue: the tail of a row-parallel linear after
    its partial accumulators are summed over ranks."""
    _require_cuda(acc, sa, wscale, bias, residual)
    m, n = acc.shape
    epi = L.EPI_RESIDUAL if residual is not None else L.EPI_NONE
    if out is None:
        out = torch.empty((m, n), dtype=torch.float16 if residual is not None else out_dtype, device=acc.device)
    L.check(L.lib.npl_dequant(acc.data_ptr(), acc.stride(0), sa.data_ptr(), wscale.data_ptr(), L.ptr(bias), m, n,
                              epi, L.ptr(residual), 0 if residual is None else residual.stride(0), out.data_ptr(),
                              out.stride(0), _DT[out.dtype], L.stream_ptr(acc.device)))
    return out


def per_output_weight_quant(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w8a8.py:53-62 (per_output_weight_qdq): (qweight int8 [N, K], scales fp32 [N])."""
    if weight.dim() < 2:
        raise ValueError("weight must have at least two dimensions")
    w = _as_f16_or_f32(weight.detach()).reshape(weight.shape[0], -1)
    k = w.shape[1]
    q, s = dynamic_per_token_quant(_pad_cols(w))
    return q[:, :k].reshape(weight.shape), s.reshape(-1)


def linear_workspace(device: torch.device, m: int, n: int, k: int) -> torch.Tensor:
    nbytes = int(L.lib.npl_linear_workspace_bytes(m, n, k))
    return L.workspaces.get(device, "linear", nbytes)


def linear_q(qa: torch.Tensor, sa: torch.Tensor, qweight: torch.Tensor, wscale: torch.Tensor, *,
             bias: torch.Tensor | None = None, epilogue: int = L.EPI_NONE,
             residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.float16, acc_out: torch.Tensor | None = None) -> torch.Tensor:
    """int8 activations [M, K] (+ per-row fp32 scales) x int8 weight [N, K].

    epilogue NONE -> [M, N] out_dtype; RESIDUAL -> fp16(fp16(v) + residual);
    SILU_MUL (qweight rows interleaved by 8, see pack_gate_up) -> [M, N/2] fp16.
    """
    _require_cuda(qa, sa, qweight, wscale, bias, residual)
    m, k = qa.shape
    n = qweight.shape[0]
    if qweight.shape[1] != k:
        raise ValueError("linear input/weight shapes do not match")
    cols = n // 2 if epilogue == L.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((m, cols), dtype=torch.float16 if epilogue else out_dtype, device=qa.device)
    if m == 0:  # nothing to launch (an empty tensor may have no device address)
        return out
    ws = linear_workspace(qa.device, m, n, k)
    res = residual
    L.check(L.lib.npl_w8a8_linear(
        qa.data_ptr(), qa.stride(0), sa.data_ptr(), qweight.data_ptr(), qweight.stride(0), wscale.data_ptr(),
        L.ptr(bias), m, n, k, epilogue, L.ptr(res), 0 if res is None else res.stride(0), out.data_ptr(),
        out.stride(0), _DT[out.dtype], L.ptr(acc_out), ws.data_ptr(), ws.numel(), L.stream_ptr(qa.device)))
    return out


def linear_ex(qweight: torch.Tensor, wscale: torch.Tensor, *, x_mode: int, m: int,
              qa: torch.Tensor | None = None, sa: torch.Tensor | None = None,
              x_f16: torch.Tensor | None = None, x_absmax: torch.Tensor | None = None,
              norm_weight: torch.Tensor | None = None, eps: float = 1e-6, bias: torch.Tensor | None = None,
              epilogue: int = L.EPI_NONE, residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.float16, acc_out: torch.Tensor | None = None,
              absmax_out: torch.Tensor | None = None, rope: dict | None = None,
              q_out: torch.Tensor | None = None, q_scale: torch.Tensor | None = None) -> torch.Tensor | None:
    """npl_w8a8_linear_ex: the decode linear with its activation preparation
    (int8 / fp16 + given absmax / fp16 + RMSNorm) and epilogue (dequant,
    residual, SiLU*up (+ absmax), RoPE + KV store) in one kernel.

    ``rope`` (for EPI_ROPE_KV): dict with cos, sin, positions, slots, q_out,
    k_cache, v_cache, heads, kv_heads, head_dim. ``q_out`` / ``q_scale`` (for
    EPI_SILU_MUL with ``absmax_out``, m <= 64): the output quantised per token
    in the same launch (int8 [m, n/2], fp32 [m]). Returns ``out`` (None for
    EPI_ROPE_KV, whose outputs are rope["q_out"] and the caches).
    """
    n, k = qweight.shape
    dev = qweight.device
    if epilogue != L.EPI_ROPE_KV and out is None:
        cols = n // 2 if epilogue == L.EPI_SILU_MUL else n
        out = torch.empty((m, cols), dtype=torch.float16 if epilogue else out_dtype, device=dev)
    a = L.NplLinearArgs()
    a.x_mode = x_mode
    if x_mode == L.X_INT8:
        a.qa, a.lda, a.sa = qa.data_ptr(), qa.stride(0), sa.data_ptr()
    else:
        a.x_f16, a.ldx = x_f16.data_ptr(), x_f16.stride(0)
        a.x_absmax = L.ptr(x_absmax)
        a.norm_weight = L.ptr(norm_weight)
        a.eps = float(eps)
    a.qw, a.ldw, a.sw, a.bias = qweight.data_ptr(), qweight.stride(0), wscale.data_ptr(), L.ptr(bias)
    a.M, a.N, a.K = m, n, k
    a.epilogue = epilogue
    if residual is not None:
        a.residual, a.ld_res = residual.data_ptr(), residual.stride(0)
    if out is not None:
        a.out, a.ld_out, a.out_dtype = out.data_ptr(), out.stride(0), _DT[out.dtype]
    a.acc_out = L.ptr(acc_out)
    a.absmax_out = L.ptr(absmax_out)
    a.q_out, a.q_scale = L.ptr(q_out), L.ptr(q_scale)
    if rope is not None:
        r = a.rope
        r.cos_table, r.sin_table = rope["cos"].data_ptr(), rope["sin"].data_ptr()
        r.max_position = rope["cos"].shape[0]
        r.positions, r.slot_mapping = rope["positions"].data_ptr(), rope["slots"].data_ptr()
        r.q_out, r.k_cache, r.v_cache = rope["q_out"].data_ptr(), rope["k_cache"].data_ptr(), rope["v_cache"].data_ptr()
        r.num_blocks, r.block_size = rope["k_cache"].shape[0], rope["k_cache"].shape[1]
        r.heads, r.kv_heads, r.head_dim = rope["heads"], rope["kv_heads"], rope["head_dim"]
    ws = linear_workspace(dev, m, n, k)
    L.check(L.lib.npl_w8a8_linear_ex(ctypes.byref(a), ws.data_ptr(), ws.numel(), L.stream_ptr(dev)))
    return out


def integer_linear_per_output(values: torch.Tensor, weight: torch.Tensor, *,
                              activation_scale: torch.Tensor | float | None = None,
                              bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """w8a8.py:118-139 on the GPU: returns (out fp32, acc int32).

    ``activation_scale`` None quantises each token with its own dynamic scale
    (the dynamic_per_token mode); a given scale (one value, or one per token)
    is used as is, as integer_linear_per_output_reference does."""
    if activation_scale is None:
        _require_cuda(values, weight)
        if values.shape[-1] != weight.shape[1] or weight.dim() != 2:
            raise ValueError("linear input/weight shapes do not match")
        k = values.shape[-1]
        qa, sa = dynamic_per_token_quant(_pad_cols(_as_f16_or_f32(values).reshape(-1, k)))
        qa, sa = qa[:, :k], sa.reshape(-1)
    else:
        return integer_linear_per_output_reference(values, weight, activation_scale=activation_scale, bias=bias)
    return _integer_linear(qa, sa, weight, bias, values.shape[:-1])


# --------------------------------------------------------------------------
# The reference's contract functions under their own names and signatures
# (w8a8.py:33-139), each running the library's kernels.
# --------------------------------------------------------------------------

def _as_f16_or_f32(values: torch.Tensor) -> torch.Tensor:
    """The kernels read fp16 or fp32; any other float type is widened to fp32
    first, exactly (the reference computes on values.float())."""
    return values if values.dtype in _DT else values.float()


def _pad_cols(t: torch.Tensor, multiple: int = 16) -> torch.Tensor:
    """[rows, K] -> [rows, ceil(K / 16) * 16] with zero columns appended (a
    zero column changes no absmax, quantises to 0 and adds 0 to every dot
    product); the kernels need 16-element rows."""
    k = t.shape[-1]
    kp = -(-k // multiple) * multiple
    if kp == k and t.stride(-1) == 1 and t.stride(0) % 16 == 0:
        return t
    out = torch.zeros((t.shape[0], kp), dtype=t.dtype, device=t.device)
    out[:, :k] = t
    return out


def _scale_operand(scale: torch.Tensor | float, rows: int, device: torch.device) -> tuple[torch.Tensor, int]:
    """A quantisation scale as the kernels take it: (fp32 [1] with stride 0)
    for one tensor-wide value, (fp32 [rows] with stride 1) for one per row."""
    s = torch.as_tensor(scale, dtype=torch.float32, device=device).detach().float()
    if bool((s <= 0).any()):  # w8a8.py:38-39
        raise ValueError("quantization scale must be positive")
    if s.numel() == 1:
        return s.reshape(1).contiguous(), 0
    if s.numel() == rows:
        return s.reshape(rows).contiguous(), 1
    raise ValueError(f"scale must hold one value or one per row ({rows}), got shape {tuple(s.shape)}")


def quantize_symmetric(values: torch.Tensor, scale: torch.Tensor | float) -> torch.Tensor:
    """w8a8.py:33-43: int8(clamp(round(values.float() / scale.float()), -127,
    127)), ties to even, one IEEE fp32 division per element. ``scale`` is one
    value or one per row of the last dimension (shape [..., 1] or [...]);
    ValueError if any scale is <= 0."""
    _require_cuda(values)
    if values.dim() == 0:
        values = values.reshape(1, 1)
    x = _as_f16_or_f32(values)
    k = x.shape[-1]
    rows = x.reshape(-1, k)
    sp, stride = _scale_operand(scale, rows.shape[0], x.device)
    xp = _pad_cols(rows)
    q = torch.empty(xp.shape, dtype=torch.int8, device=x.device)
    if rows.shape[0]:
        L.check(L.lib.npl_quant_given_scale(xp.data_ptr(), _DT[xp.dtype], xp.shape[0], xp.shape[1], xp.stride(0),
                                            sp.data_ptr(), stride, q.data_ptr(), q.stride(0), L.stream_ptr(x.device)))
    return q[:, :k].reshape(values.shape)


def scale_from_absmax(absmax: torch.Tensor) -> torch.Tensor:
    """w8a8.py:46-50: fp32(fp16(max(absmax, fp16.tiny) / 127)), >= fp16.tiny,
    elementwise (same shape as ``absmax``)."""
    _require_cuda(absmax)
    a = absmax.detach().float().contiguous()
    out = torch.empty_like(a)
    L.check(L.lib.npl_scale_from_absmax(a.data_ptr(), a.numel(), out.data_ptr(), L.stream_ptr(a.device)))
    return out


def _dequant_rows(q: torch.Tensor, scale: torch.Tensor, stride: int, dtype: torch.dtype) -> torch.Tensor:
    """fp32(q) * scale per row (npl_dequant_rows), returned as ``dtype``
    (fp16 rounded once in the kernel; other types through fp32)."""
    k = q.shape[-1]
    qp = _pad_cols(q.reshape(-1, k))
    out_dt = torch.float16 if dtype == torch.float16 else torch.float32
    out = torch.empty(qp.shape, dtype=out_dt, device=q.device)
    if qp.shape[0]:
        L.check(L.lib.npl_dequant_rows(qp.data_ptr(), qp.shape[0], qp.shape[1], qp.stride(0), scale.data_ptr(),
                                       stride, out.data_ptr(), out.stride(0), _DT[out_dt], L.stream_ptr(q.device)))
    return out[:, :k].reshape(q.shape).to(dtype)


def per_output_weight_qdq(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """w8a8.py:53-62: (dequantised weight in weight.dtype, int8 weight of the
    same shape, fp32 per-output-channel scales [N])."""
    _require_cuda(weight)
    q, s = per_output_weight_quant(weight)
    deq = _dequant_rows(q.reshape(weight.shape[0], -1), s, 1, weight.dtype)
    return deq.reshape(weight.shape), q, s


def static_activation_scale(absmax: float | torch.Tensor, device: torch.device | None = None) -> torch.Tensor:
    """w8a8.py:94-99: the tensor-wide scale of one absmax, a 0-dim fp32 CUDA
    tensor (on ``device``, or the absmax's device, or the current one)."""
    if device is None:
        device = absmax.device if isinstance(absmax, torch.Tensor) and absmax.is_cuda else \
            torch.device("cuda", torch.cuda.current_device())
    value = torch.as_tensor(absmax, dtype=torch.float32, device=device)
    if value.numel() != 1:
        raise ValueError("static activation scale expects one tensor-wide absmax")
    return scale_from_absmax(value.reshape(()))


def static_activation_qdq(values: torch.Tensor, scale: torch.Tensor | float) -> torch.Tensor:
    """w8a8.py:101-103: quantise with the given scale and dequantise, in
    values.dtype."""
    q = quantize_symmetric(values, scale)
    k = q.shape[-1] if q.dim() else 1
    sp, stride = _scale_operand(scale, q.numel() // max(1, k), values.device)
    return _dequant_rows(q.reshape(-1, k), sp, stride, values.dtype).reshape(values.shape)


def dynamic_per_token_activation_qdq(values: torch.Tensor, *, axis: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    """w8a8.py:106-115: (QDQ values in values.dtype, fp32 scales with the
    reduced axis kept as size 1), one scale per slice along ``axis``."""
    if values.dim() == 0:
        raise ValueError("dynamic per-token quantization expects a tensor")
    _require_cuda(values)
    ax = axis % values.dim()
    v = values.movedim(ax, -1)
    k = v.shape[-1]
    rows = _pad_cols(_as_f16_or_f32(v).reshape(-1, k))
    q, s = dynamic_per_token_quant(rows)
    s = s.reshape(-1)
    deq = _dequant_rows(q[:, :k], s, 1, values.dtype).reshape(v.shape).movedim(-1, ax)
    return deq, s.reshape(*v.shape[:-1], 1).movedim(-1, ax)


def _integer_linear(qa: torch.Tensor, sa: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                    lead: torch.Size) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 activations [rows, K] + fp32 per-row scales x the per-output
    quantised ``weight`` -> (out fp32, acc int32) shaped [*lead, N]."""
    qw, sw = per_output_weight_quant(weight)
    k = qw.shape[1]
    qa2 = _pad_cols(qa.reshape(-1, k))
    qw = _pad_cols(qw)
    acc = torch.empty((qa2.shape[0], qw.shape[0]), dtype=torch.int32, device=qw.device)
    b = None if bias is None else bias.detach().float().contiguous()
    out = linear_q(qa2, sa.contiguous(), qw, sw, bias=b, out_dtype=torch.float32, acc_out=acc)
    return out.reshape(*lead, qw.shape[0]), acc.reshape(*lead, qw.shape[0])


def integer_linear_per_output_reference(values: torch.Tensor, weight: torch.Tensor, *,
                                        activation_scale: torch.Tensor | float,
                                        bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """w8a8.py:118-139 with its signature, on the GPU: int8 activations from
    ``activation_scale`` (one tensor-wide value -- the static mode -- or one
    per token), per-output-channel int8 weights, int8 x int8 -> int32 on the
    tensor cores, then ((acc * s_a) * s_w) + bias in fp32. Returns (out fp32,
    acc int32), both [..., N]."""
    _require_cuda(values, weight)
    if values.shape[-1] != weight.shape[1] or weight.dim() != 2:
        raise ValueError("linear input/weight shapes do not match")
    qa = quantize_symmetric(values, activation_scale)
    rows = qa.numel() // max(1, qa.shape[-1]) if qa.dim() else 1
    sp, stride = _scale_operand(activation_scale, rows, values.device)
    sa = sp.expand(rows) if stride == 0 else sp
    return _integer_linear(qa, sa, weight, bias, values.shape[:-1])


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``act_fn(gate) * up`` of the unfused MLP on fp16 values
    (lightweight_runner.py:358): fp16(fp16(silu(gate)) * up), SiLU rounded
    once to fp16 from the exact value (npl_silu_mul, the arithmetic of the
    SiLU * up epilogue)."""
    _require_cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != torch.float16 or up.dtype != torch.float16:
        raise ValueError("silu_mul: gate and up must be fp16 tensors of one shape")
    cols = gate.shape[-1] if gate.dim() else 1
    g = _pad_cols(gate.reshape(-1, cols), 8)
    u = _pad_cols(up.reshape(-1, cols), 8)
    out = torch.empty_like(g)
    if g.shape[0]:
        L.check(L.lib.npl_silu_mul(g.data_ptr(), g.stride(0), u.data_ptr(), u.stride(0), g.shape[0], g.shape[1],
                                   out.data_ptr(), out.stride(0), L.stream_ptr(gate.device)))
    return out[:, :cols].reshape(gate.shape)


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Row layout the SiLU*up epilogue reads: groups of 16 rows, group j
    holding gate rows [8j, 8j+8) followed by up rows [8j, 8j+8), so that a
    128-row weight tile carries the gate and up rows of 64 outputs and one
    16x256b TMEM load hands each epilogue thread a gate row together with its
    up row. Works on weights [I, K] or per-row scales [I]; I must be a
    multiple of 64 (whole 128-row tiles)."""
    inter = gate.shape[0]
    if inter % 64 or up.shape != gate.shape:
        raise ValueError("gate/up must match and have a multiple of 64 rows")
    g = gate.reshape(inter // 8, 8, *gate.shape[1:])
    u = up.reshape(inter // 8, 8, *up.shape[1:])
    return torch.stack([g, u], dim=1).reshape(2 * inter, *gate.shape[1:]).contiguous()


class W8A8Linear:
    """A quantised Linear: int8 weight [N, K] (row-major, K contiguous) with
    per-output-channel fp32 scales (fp16 values) and an optional fp32 bias.

    The drop-in for the reference's ``nn.Linear`` under W8A8 (weights from
    per_output_weight_qdq, activations from dynamic per-token quantisation).
    """

    def __init__(self, qweight: torch.Tensor, wscale: torch.Tensor, bias: torch.Tensor | None = None, *,
                 activation_scale: torch.Tensor | float | None = None):
        """``activation_scale``: None quantises each call's tokens with their
        own dynamic scales (dynamic_per_token, w8a8.py:106-115); a given
        tensor-wide value is the static mode (w8a8.py:94-103)."""
        if qweight.dtype != torch.int8 or qweight.dim() != 2:
            raise ValueError("qweight must be int8 [N, K]")
        self.qweight = qweight.contiguous()
        self.wscale = wscale.float().contiguous()
        self.bias = None if bias is None else bias.float().contiguous()
        self.activation_scale = None
        if activation_scale is not None:
            s = torch.as_tensor(activation_scale, dtype=torch.float32, device=self.qweight.device)
            if s.numel() != 1 or float(s) <= 0:
                raise ValueError("a static activation scale is one positive value")
            self.activation_scale = s.reshape(1).contiguous()

    @classmethod
    def from_float(cls, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
                   activation_scale: torch.Tensor | float | None = None) -> "W8A8Linear":
        q, s = per_output_weight_quant(weight)
        return cls(q, s, bias, activation_scale=activation_scale)

    @property
    def out_features(self) -> int:
        return self.qweight.shape[0]

    @property
    def in_features(self) -> int:
        return self.qweight.shape[1]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.activation_scale is None:
            qa, sa = dynamic_per_token_quant(x)
        else:
            qa = quantize_symmetric(x, self.activation_scale)
            sa = self.activation_scale.expand(qa.numel() // x.shape[-1]).contiguous()
        out = linear_q(qa.reshape(-1, x.shape[-1]), sa.reshape(-1), self.qweight, self.wscale, bias=self.bias,
                       out_dtype=torch.float16 if x.dtype == torch.float16 else torch.float32)
        return out.reshape(*x.shape[:-1], self.out_features)
