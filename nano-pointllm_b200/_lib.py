"""ctypes binding of libnpl_w8a8.so (the C ABI declared in include/npl_w8a8.h).

The library is built in-tree by ``build.py``; importing this module loads it
and fails loudly when it is missing: there is no fallback implementation.
Status codes map to the exceptions the reference raises for the same
conditions (w8a8.py:38-39,126-127: ValueError; :152-153: OverflowError).
"""
from __future__ import annotations

import ctypes
import pathlib

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libnpl_w8a8.so"

NPL_OK = 0
NPL_ERR_ARG = 1
NPL_ERR_OVERFLOW = 2
NPL_ERR_LAUNCH = 3
NPL_ERR_TIMEOUT = 4
NPL_ERR_UNSUPPORTED = 5

NPL_F32 = 0
NPL_F16 = 1

EPI_NONE = 0
EPI_RESIDUAL = 1
EPI_SILU_MUL = 2
EPI_ROPE_KV = 3

X_INT8 = 0
X_F16_ABSMAX = 1
X_F16_RMSNORM = 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t

class NplRopeKV(ctypes.Structure):
    """npl_rope_kv (include/npl_w8a8.h)."""
    _fields_ = [("cos_table", _P), ("sin_table", _P), ("max_position", _I), ("positions", _P),
                ("slot_mapping", _P), ("q_out", _P), ("k_cache", _P), ("v_cache", _P), ("num_blocks", _I),
                ("block_size", _I), ("heads", _I), ("kv_heads", _I), ("head_dim", _I)]


class NplLinearArgs(ctypes.Structure):
    """npl_linear_args (include/npl_w8a8.h)."""
    _fields_ = [("x_mode", _I), ("qa", _P), ("lda", _I), ("sa", _P), ("x_f16", _P), ("ldx", _I),
                ("x_absmax", _P), ("norm_weight", _P), ("eps", _F), ("qw", _P), ("ldw", _I), ("sw", _P),
                ("bias", _P), ("M", _I), ("N", _I), ("K", _I), ("epilogue", _I), ("residual", _P), ("ld_res", _I),
                ("out", _P), ("ld_out", _I), ("out_dtype", _I), ("acc_out", _P), ("absmax_out", _P),
                ("rope", NplRopeKV), ("q_out", _P), ("q_scale", _P)]


TP_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class NplTpPeers(ctypes.Structure):
    """npl_tp_peers (include/npl_w8a8.h)."""
    _fields_ = [("world", _I), ("rank", _I), ("buffers", _P * TP_MAX_RANKS), ("max_elems", ctypes.c_longlong)]


# name -> (restype, argtypes); mirrors include/npl_w8a8.h
SIGNATURES = {
    "npl_last_error_string": (ctypes.c_char_p, []),
    "npl_version": (_I, []),
    "npl_device_status": (_I, [ctypes.POINTER(_I), _I]),
    "npl_quant_rows": (_I, [_P, _I, _I, _I, _I, _P, _I, _P, _P]),
    "npl_row_absmax": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "npl_quant_rows_absmax": (_I, [_P, _I, _I, _I, _I, _P, _P, _I, _P, _P]),
    "npl_quant_given_scale": (_I, [_P, _I, _I, _I, _I, _P, _I, _P, _I, _P]),
    "npl_dequant_rows": (_I, [_P, _I, _I, _I, _P, _I, _P, _I, _I, _P]),
    "npl_scale_from_absmax": (_I, [_P, _I, _P, _P]),
    "npl_silu_mul": (_I, [_P, _I, _P, _I, _I, _I, _P, _I, _P]),
    "npl_dequant": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _P, _I, _P, _I, _I, _P]),
    "npl_rmsnorm_quant": (_I, [_P, _P, _P, _F, _I, _I, _P, _P, _P, _P, _P]),
    "npl_linear_workspace_bytes": (_Z, [_I, _I, _I]),
    "npl_w8a8_linear": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _P, _I, _I, _P, _P, _Z, _P]),
    "npl_w8a8_linear_ex": (_I, [ctypes.POINTER(NplLinearArgs), _P, _Z, _P]),
    "npl_w8a8_linear_noalloc": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _P, _I, _I, _P, _P]),
    "npl_store_kv": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _I, _I, _P]),
    "npl_rope_store_kv": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _P]),
    "npl_decode_attention_workspace_bytes": (_Z, [_I, _I, _I, _I, _I]),
    "npl_paged_decode_attention": (_I, [_P, _I, _I, _I, _I, _P, _P, _I, _I, _P, _I, _I, _P, _F, _P, _P, _P, _P, _Z,
                                        _P]),
    "npl_tp_exchange_bytes": (_Z, [_I, ctypes.c_longlong]),
    "npl_ipc_handle": (_I, [_P, _P, ctypes.POINTER(_Z)]),
    "npl_ipc_open": (_I, [_P, _Z, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "npl_ipc_close": (_I, [_P]),
    "npl_tp_absmax_quant": (_I, [ctypes.POINTER(NplTpPeers), _P, _I, _I, _I, _P, _I, _P, _P]),
    "npl_tp_allreduce_dequant": (_I, [ctypes.POINTER(NplTpPeers), _P, _I, _I, _P, _P, _P, _P, _I, _P, _I, _P]),
    "npl_paged_prefill_attention": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _I, _I, _F,
                                         _P, _I, _P]),
}


class NplError(RuntimeError):
    pass


class NplTimeout(NplError):
    pass


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python nano-pointllm_b200/build.py` "
            "(the W8A8 path has no fallback implementation)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc: int) -> None:
    if rc == NPL_OK:
        return
    msg = lib.npl_last_error_string().decode(errors="replace")
    if rc == NPL_ERR_ARG:
        raise ValueError(msg)
    if rc == NPL_ERR_OVERFLOW:
        raise OverflowError(msg)
    if rc == NPL_ERR_TIMEOUT:
        raise NplTimeout(msg)
    raise NplError(f"[{rc}] {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(reset: bool = True) -> int:
    """Reads (and by default clears) the device status word of the current
    device; raises NplTimeout if a kernel gave up a bounded wait."""
    code = _I(0)
    rc = lib.npl_device_status(ctypes.byref(code), 1 if reset else 0)
    if rc != NPL_OK and code.value == 0:
        check(rc)
    if code.value:
        raise NplTimeout(f"device status word = {code.value}")
    return 0


class Workspaces:
    """Zero-initialised device scratch buffers, one per (device, tag), grown
    on demand. Kernels leave them zeroed, so they are allocated and cleared
    once; allocate the largest size before CUDA-graph capture."""

    def __init__(self) -> None:
        self._bufs: dict[tuple[int, str], torch.Tensor] = {}

    def get(self, device: torch.device, tag: str, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), tag)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"workspace '{tag}' must be sized before CUDA graph capture")
            buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


workspaces = Workspaces()
