"""Checksummed int8 weight packages: quantise once, start from the int8 bytes.

Two package kinds share one directory schema (schema_version "1.0"): a
``metadata.json`` manifest plus one raw little-endian, row-major file per
tensor, each described by ``{file, dtype, shape, order, bytes, sha256}``.

* The single-linear package of the reference
  (nanopointllm/compression/quantized_tensor_package.py:46-186): int8
  activation [M, K] and weight [N, K], fp16 per-tensor activation scale,
  per-output weight scales, SmoothQuant scales, optional output scale and
  bias. ``write_quantized_linear_package`` writes the same bytes as the
  reference's writer for the same inputs (manifest and tensor files), and
  ``load_quantized_linear_package`` reads packages written by either. The
  integer golden A @ W^T (quantized_tensor_package.py:39-43) runs on the GPU
  through npl_w8a8_linear's int32 accumulator output.
* The whole-model package of W8A8LlamaRunner: for every Linear of the Llama
  (q/k/v/o/gate/up/down per layer and the LM head) its int8 weight [N, K]
  and fp16 per-output scales; the embedding and RMSNorm weights as fp16; the
  model geometry and the numerical contract in the manifest. A runner built
  from it (``W8A8LlamaRunner.from_package``) skips the per-output
  quantisation of every weight at start-up and is bit-identical to one built
  from the float weights.

Every tensor is checked before it is exposed: the manifest is validated in
full (schema, package type, the exact tensor set, each dtype/shape against
the geometry, file names without directories) before any data is read, and
each file's byte count and SHA-256 before its bytes are used. Loading runs
on a thread pool ahead of use: each large tensor is read in 16 MB chunks
into reused pinned buffers, hashed there and copied to the GPU on the
thread's own stream while the next chunk is read (fresh host allocations
would cost more than the reads themselves: first-touch page faults), and
the device tensor is handed out only after the whole file's hash matched.
"""
from __future__ import annotations

import hashlib
import json
import os
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, fields
from pathlib import Path
from typing import Any, Mapping

import numpy as np
import torch

from .synthetic import LlamaShape

SCHEMA_VERSION = "1.0"
LINEAR_PACKAGE_TYPE = "smoothquant_static_a8_per_output_w8_linear"
LLAMA_PACKAGE_TYPE = "w8a8_dynamic_per_token_a8_per_output_w8_llama"
MANIFEST = "metadata.json"

_INT8 = np.dtype("i1")
_FP16 = np.dtype("<f2")

LINEAR_CONTRACT = {
    "activation": "symmetric_per_tensor_int8[-127,127]",
    "weight": "symmetric_per_output_int8[-127,127]",
    "scale_storage": "IEEE754_binary16_little_endian",
    "accumulator": "signed_int32",
    "rounding": "round_to_nearest_ties_to_even",
    "layout": "row_major",
}

LLAMA_CONTRACT = {
    "activation": "symmetric_dynamic_per_token_int8[-127,127]",
    "weight": "symmetric_per_output_int8[-127,127]",
    "scale_storage": "IEEE754_binary16_little_endian",
    "accumulator": "signed_int32",
    "rounding": "round_to_nearest_ties_to_even",
    "layout": "row_major",
    "norm_residual": "float16",
}


# ------------------------------------------------------------------ tensor files
def _entry(filename: str, array: np.ndarray, payload: bytes | memoryview) -> dict[str, Any]:
    return {
        "file": filename,
        "dtype": array.dtype.str,
        "shape": [int(d) for d in array.shape],
        "order": "C",
        "bytes": len(payload),
        "sha256": hashlib.sha256(payload).hexdigest(),
    }


def _write_tensor(root: Path, filename: str, array: np.ndarray) -> dict[str, Any]:
    array = np.ascontiguousarray(array)
    payload = memoryview(array).cast("B")
    with open(root / filename, "wb") as f:
        f.write(payload)
    return _entry(filename, array, payload)


def _write_manifest(root: Path, manifest: dict[str, Any]) -> None:
    text = json.dumps(manifest, indent=2, sort_keys=True) + "\n"
    tmp = root / (MANIFEST + ".tmp")
    tmp.write_text(text, encoding="utf-8")
    os.replace(tmp, root / MANIFEST)  # the manifest appears only once every file is written


def _read_manifest(root: Path) -> dict[str, Any]:
    manifest = json.loads((root / MANIFEST).read_text(encoding="utf-8"))
    if not isinstance(manifest, dict) or manifest.get("schema_version") != SCHEMA_VERSION:
        raise ValueError("unsupported quantized tensor package schema")
    if not isinstance(manifest.get("tensors"), dict):
        raise ValueError("package manifest has no tensor table")
    return manifest


def _check_entry_meta(name: str, entry: Any, dtype: np.dtype | None = None,
                      shape: tuple[int, ...] | None = None) -> tuple[np.dtype, tuple[int, ...]]:
    """Validates one manifest entry without touching its file."""
    if not isinstance(entry, dict):
        raise ValueError(f"{name}: malformed manifest entry")
    fname = entry.get("file")
    if not isinstance(fname, str) or not fname or fname in (".", "..") or "/" in fname or "\\" in fname:
        raise ValueError(f"{name}: tensor file must be a plain file name inside the package")
    if entry.get("order", "C") != "C":
        raise ValueError(f"{name}: only row-major ('C') tensors are supported")
    try:
        dt = np.dtype(entry["dtype"])
        shp = tuple(int(v) for v in entry["shape"])
        nbytes = int(entry["bytes"])
    except (KeyError, TypeError, ValueError) as e:
        raise ValueError(f"{name}: malformed manifest entry ({e})") from None
    digest = entry.get("sha256")
    if not isinstance(digest, str) or len(digest) != 64:
        raise ValueError(f"{name}: manifest entry has no SHA256")
    if any(d < 0 for d in shp):
        raise ValueError(f"{name}: negative dimension")
    if int(np.prod(shp, dtype=np.int64)) * dt.itemsize != nbytes:
        raise ValueError(f"{name} metadata size mismatch")
    if dtype is not None and dt != dtype:
        raise ValueError(f"{name}: dtype {dt.str} where {np.dtype(dtype).str} is required")
    if shape is not None and shp != tuple(shape):
        raise ValueError(f"{name}: shape {list(shp)} where {list(shape)} is required")
    return dt, shp


def _read_verified(root: Path, name: str, entry: dict[str, Any]) -> np.ndarray:
    """The tensor's bytes, after the byte count and the SHA-256 check."""
    dt, shp = _check_entry_meta(name, entry)
    nbytes = int(entry["bytes"])
    path = root / entry["file"]
    buf = bytearray(nbytes)
    with open(path, "rb") as f:
        got = f.readinto(buf)
        extra = f.read(1)
    if got != nbytes or extra:
        raise ValueError(f"{name} byte count mismatch")
    if hashlib.sha256(buf).hexdigest() != entry["sha256"]:
        raise ValueError(f"{name} SHA256 mismatch")
    return np.frombuffer(buf, dtype=dt).reshape(shp)


_TORCH_DTYPE = {_INT8: torch.int8, _FP16: torch.float16}
STAGING_CHUNK = 16 << 20   # bytes per pinned staging buffer (two per loader thread)
DEVICE_MIN_BYTES = 1 << 20  # smaller tensors take the host path


class _Staging:
    """Two pinned host buffers and a copy stream: one loader thread reads and
    hashes into one buffer while the other is being copied to the device."""

    def __init__(self, device: torch.device, chunk: int):
        self.bufs = [torch.empty(chunk, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.views = [b.numpy() for b in self.bufs]
        self.events = [torch.cuda.Event() for _ in range(2)]
        self.stream = torch.cuda.Stream(device=device)


def _read_verified_to_device(root: Path, name: str, entry: dict[str, Any], device: torch.device,
                             staging: _Staging) -> torch.Tensor:
    """Streams one tensor file to the device through the pinned buffers,
    hashing each chunk on the way. The device tensor is returned only when
    the byte count and the SHA-256 of everything copied match the manifest."""
    dt, shp = _check_entry_meta(name, entry)
    nbytes = int(entry["bytes"])
    out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    digest = hashlib.sha256()
    chunk = staging.views[0].shape[0]
    with open(root / entry["file"], "rb", buffering=0) as f:
        if os.fstat(f.fileno()).st_size != nbytes:
            raise ValueError(f"{name} byte count mismatch")
        with torch.cuda.stream(staging.stream):
            off, i = 0, 0
            while off < nbytes:
                k = i & 1
                staging.events[k].synchronize()  # the previous copy out of this buffer is done
                n = min(chunk, nbytes - off)
                view = staging.views[k][:n]
                got = 0
                while got < n:
                    r = f.readinto(view[got:])
                    if not r:
                        raise ValueError(f"{name} byte count mismatch")
                    got += r
                digest.update(view)
                out[off:off + n].copy_(staging.bufs[k][:n], non_blocking=True)
                staging.events[k].record(staging.stream)
                off += n
                i += 1
        if f.read(1):
            raise ValueError(f"{name} byte count mismatch")
    staging.stream.synchronize()
    if digest.hexdigest() != entry["sha256"]:
        raise ValueError(f"{name} SHA256 mismatch")
    return out.view(_TORCH_DTYPE[dt]).reshape(shp)


def _canonical(values: Any, dtype: np.dtype, name: str, *, dimensions: int) -> np.ndarray:
    array = values.detach().cpu().numpy() if isinstance(values, torch.Tensor) else np.asarray(values)
    if array.ndim != dimensions:
        raise ValueError(f"{name} must have {dimensions} dimensions")
    if array.dtype.kind == "f" and not np.all(np.isfinite(array)):
        raise ValueError(f"{name} contains non-finite values")
    return np.ascontiguousarray(array.astype(dtype, copy=False))


# ---------------------------------------------------------- single-linear package
@dataclass(frozen=True)
class QuantizedLinearTensors:
    """One quantised linear (quantized_tensor_package.py:16-43)."""
    activation: np.ndarray
    weight: np.ndarray
    activation_scale: np.ndarray
    weight_scale: np.ndarray
    smooth_scale: np.ndarray
    output_scale: np.ndarray | None
    bias: np.ndarray | None
    metadata: dict[str, Any]

    @property
    def m(self) -> int:
        return int(self.activation.shape[0])

    @property
    def n(self) -> int:
        return int(self.weight.shape[0])

    @property
    def k(self) -> int:
        return int(self.weight.shape[1])

    def integer_golden(self, device: torch.device | str = "cuda") -> np.ndarray:
        """activation @ weight^T in int32, computed by the tcgen05 linear
        (its int32 accumulator output). K is zero-padded to the kernel's
        multiple of 16, which adds nothing to any sum."""
        from . import w8a8 as W
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("integer_golden runs on a CUDA device")
        kp = -(-self.k // 16) * 16
        a = torch.zeros((self.m, kp), dtype=torch.int8, device=dev)
        w = torch.zeros((self.n, kp), dtype=torch.int8, device=dev)
        a[:, :self.k] = torch.from_numpy(np.ascontiguousarray(self.activation)).to(dev)
        w[:, :self.k] = torch.from_numpy(np.ascontiguousarray(self.weight)).to(dev)
        sa = torch.full((self.m,), float(self.activation_scale.reshape(-1)[0]), dtype=torch.float32, device=dev)
        sw = torch.from_numpy(self.weight_scale.astype(np.float32)).to(dev)
        acc = torch.empty((self.m, self.n), dtype=torch.int32, device=dev)
        if self.m:
            W.linear_q(a, sa, w, sw, acc_out=acc)
        return acc.cpu().numpy()


def write_quantized_linear_package(directory: str | Path, *, activation, weight, activation_scale,
                                   weight_scale, smooth_scale, output_scale=None, bias=None,
                                   provenance: dict[str, Any] | None = None) -> dict[str, Any]:
    """Writes one row-major linear package and returns its manifest
    (quantized_tensor_package.py:46-140: same files, same manifest bytes)."""
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    activation = _canonical(activation, _INT8, "activation", dimensions=2)
    weight = _canonical(weight, _INT8, "weight", dimensions=2)
    if activation.shape[1] != weight.shape[1]:
        raise ValueError("activation and weight K dimensions differ")
    activation_scale = _canonical(np.asarray(activation_scale).reshape(-1), _FP16, "activation_scale", dimensions=1)
    if activation_scale.shape != (1,):
        raise ValueError("activation_scale must contain exactly one FP16 value")
    weight_scale = _canonical(weight_scale, _FP16, "weight_scale", dimensions=1)
    smooth_scale = _canonical(smooth_scale, _FP16, "smooth_scale", dimensions=1)
    if weight_scale.shape != (weight.shape[0],):
        raise ValueError("weight_scale must contain one value per output")
    if smooth_scale.shape != (weight.shape[1],):
        raise ValueError("smooth_scale must contain one value per input channel")
    if np.any(activation_scale <= 0) or np.any(weight_scale <= 0):
        raise ValueError("quantization scales must be positive")
    if np.any(smooth_scale <= 0):
        raise ValueError("SmoothQuant scales must be positive")
    tensors = {
        "activation": ("activation.int8", activation),
        "weight": ("weight.int8", weight),
        "activation_scale": ("activation_scale.fp16", activation_scale),
        "weight_scale": ("weight_scale.fp16", weight_scale),
        "smooth_scale": ("smooth_scale.fp16", smooth_scale),
    }
    if output_scale is not None:
        out_s = _canonical(np.asarray(output_scale).reshape(-1), _FP16, "output_scale", dimensions=1)
        if out_s.shape != (1,) or np.any(out_s <= 0):
            raise ValueError("output_scale must contain one positive FP16 value")
        tensors["output_scale"] = ("output_scale.fp16", out_s)
    if bias is not None:
        b = _canonical(bias, _FP16, "bias", dimensions=1)
        if b.shape != (weight.shape[0],):
            raise ValueError("bias must contain one value per output")
        tensors["bias"] = ("bias.fp16", b)
    entries = {name: _write_tensor(root, fname, arr) for name, (fname, arr) in tensors.items()}
    manifest = {
        "schema_version": SCHEMA_VERSION,
        "package_type": LINEAR_PACKAGE_TYPE,
        "shape": {"m": int(activation.shape[0]), "n": int(weight.shape[0]), "k": int(weight.shape[1])},
        "numerical_contract": dict(LINEAR_CONTRACT),
        "tensors": entries,
        "provenance": provenance or {},
    }
    _write_manifest(root, manifest)
    return manifest


def load_quantized_linear_package(directory: str | Path) -> QuantizedLinearTensors:
    """Loads and validates a linear package before exposing any array
    (quantized_tensor_package.py:143-186)."""
    root = Path(directory)
    manifest = _read_manifest(root)
    entries = manifest["tensors"]
    required = {"activation", "weight", "activation_scale", "weight_scale", "smooth_scale"}
    missing = sorted(required - set(entries))
    if missing:
        raise ValueError(f"quantized tensor package is missing {missing}")
    arrays = {name: _read_verified(root, name, entry).copy() for name, entry in entries.items()}
    try:
        m, n, k = (int(manifest["shape"][d]) for d in ("m", "n", "k"))
    except (KeyError, TypeError, ValueError):
        raise ValueError("package manifest has no m/n/k shape") from None
    if arrays["activation"].shape != (m, k):
        raise ValueError("activation shape does not match package shape")
    if arrays["weight"].shape != (n, k):
        raise ValueError("weight shape does not match package shape")
    if arrays["activation_scale"].shape != (1,):
        raise ValueError("activation_scale shape must be [1]")
    if arrays["weight_scale"].shape != (n,):
        raise ValueError("weight_scale shape does not match N")
    if arrays["smooth_scale"].shape != (k,):
        raise ValueError("smooth_scale shape does not match K")
    output_scale, bias = arrays.get("output_scale"), arrays.get("bias")
    if output_scale is not None and output_scale.shape != (1,):
        raise ValueError("output_scale shape must be [1]")
    if bias is not None and bias.shape != (n,):
        raise ValueError("bias shape does not match N")
    return QuantizedLinearTensors(activation=arrays["activation"], weight=arrays["weight"],
                                  activation_scale=arrays["activation_scale"], weight_scale=arrays["weight_scale"],
                                  smooth_scale=arrays["smooth_scale"], output_scale=output_scale, bias=bias,
                                  metadata=manifest)


# ------------------------------------------------------------ Llama weight sources
def llama_linear_modules(shape: LlamaShape) -> list[tuple[str, int, int]]:
    """(module, N, K) of every Linear, in the order the runner builds them."""
    h, i_, d = shape.hidden, shape.intermediate, shape.head_dim
    q, kv = shape.heads * d, shape.kv_heads * d
    mods = []
    for layer in range(shape.layers):
        p = f"model.layers.{layer}."
        mods += [(p + "self_attn.q_proj", q, h), (p + "self_attn.k_proj", kv, h), (p + "self_attn.v_proj", kv, h),
                 (p + "self_attn.o_proj", h, q), (p + "mlp.gate_proj", i_, h), (p + "mlp.up_proj", i_, h),
                 (p + "mlp.down_proj", h, i_)]
    return mods + [("lm_head", shape.vocab, h)]


def llama_dense_tensors(shape: LlamaShape) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of the fp16 tensors that stay unquantised."""
    h = shape.hidden
    names = [("model.embed_tokens.weight", (shape.vocab, h))]
    for layer in range(shape.layers):
        p = f"model.layers.{layer}."
        names += [(p + "input_layernorm.weight", (h,)), (p + "post_attention_layernorm.weight", (h,))]
    return names + [("model.norm.weight", (h,))]


class FloatLlamaWeights:
    """Weight source over an HF-named float state dict: each Linear is
    quantised per output channel on the GPU (npl_quant_rows) when the runner
    asks for it, so the fp16 weights are never all on the device at once."""

    def __init__(self, state_dict: Mapping[str, torch.Tensor], device: torch.device | str):
        self.sd = state_dict
        self.device = torch.device(device)

    def linear(self, module: str) -> tuple[torch.Tensor, torch.Tensor]:
        from . import w8a8 as W
        return W.per_output_weight_quant(self.sd[module + ".weight"].to(device=self.device, dtype=torch.float16))

    def dense(self, name: str) -> torch.Tensor:
        return self.sd[name].to(device=self.device, dtype=torch.float16).contiguous()


def as_weight_source(weights: Any, device: torch.device | str):
    """A runner's weights: a source with linear()/dense(), or a float state dict."""
    if hasattr(weights, "linear") and hasattr(weights, "dense"):
        return weights
    return FloatLlamaWeights(weights, device)


def _shape_from_manifest(manifest: dict[str, Any]) -> LlamaShape:
    raw = manifest.get("llama_shape")
    if not isinstance(raw, dict):
        raise ValueError("package manifest has no llama_shape")
    names = {f.name for f in fields(LlamaShape)}
    if set(raw) != names:
        raise ValueError(f"llama_shape must name exactly {sorted(names)}")
    ints = {"hidden", "heads", "kv_heads", "head_dim", "intermediate", "layers", "vocab", "max_position"}
    try:
        vals = {k: (int(v) if k in ints else float(v)) for k, v in raw.items()}
    except (TypeError, ValueError):
        raise ValueError("llama_shape holds a non-numeric value") from None
    shape = LlamaShape(**vals)
    if min(shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.intermediate, shape.layers,
           shape.vocab) <= 0 or shape.heads % shape.kv_heads:
        raise ValueError("llama_shape is not a valid geometry")
    return shape


def _llama_expected(shape: LlamaShape) -> dict[str, tuple[np.dtype, tuple[int, ...]]]:
    want: dict[str, tuple[np.dtype, tuple[int, ...]]] = {}
    for mod, n, k in llama_linear_modules(shape):
        want[mod + ".weight"] = (_INT8, (n, k))
        want[mod + ".weight_scale"] = (_FP16, (n,))
    for name, shp in llama_dense_tensors(shape):
        want[name] = (_FP16, shp)
    return want


class PackagedLlamaWeights:
    """Weight source over a whole-model package. The constructor validates the
    manifest in full; tensors are read, byte-counted and SHA-256-checked on a
    thread pool ahead of use (``read_ahead_bytes`` bounds the bytes held),
    and each reaches the GPU only after its check passed."""

    def __init__(self, directory: str | Path, device: torch.device | str, *, threads: int = 8,
                 read_ahead_bytes: int = 2 << 30):
        self.root = Path(directory)
        self.device = torch.device(device)
        self._staging: list[_Staging] = []  # free staging sets (CUDA devices only)
        self.manifest = _read_manifest(self.root)
        if self.manifest.get("package_type") != LLAMA_PACKAGE_TYPE:
            raise ValueError(f"not a W8A8 Llama package (package_type {self.manifest.get('package_type')!r})")
        self.shape = _shape_from_manifest(self.manifest)
        entries = self.manifest["tensors"]
        want = _llama_expected(self.shape)
        missing, extra = sorted(set(want) - set(entries)), sorted(set(entries) - set(want))
        if missing:
            raise ValueError(f"W8A8 Llama package is missing {missing[:4]}{' ...' if len(missing) > 4 else ''}")
        if extra:
            raise ValueError(f"W8A8 Llama package holds unexpected tensors {extra[:4]}")
        files = set()
        for name, (dt, shp) in want.items():
            _check_entry_meta(name, entries[name], dt, shp)
            files.add(entries[name]["file"])
        if len(files) != len(want):
            raise ValueError("two package tensors share one file")
        # read-ahead in the runner's order of use
        self._order = sorted(want, key=self._use_rank)
        self._want = set(want)
        self._pool = ThreadPoolExecutor(max_workers=max(1, threads), thread_name_prefix="npl-pkg")
        self._futures: dict[str, tuple[Future, int]] = {}
        self._taken: set[str] = set()
        self._inflight = 0
        self._budget = int(read_ahead_bytes)
        self._next = 0
        self._pump()

    @staticmethod
    def _use_rank(name: str) -> tuple[int, int, str]:
        """The runner asks for the embedding, then layer by layer, then the
        final norm and the LM head."""
        if name.startswith("model.embed_tokens"):
            return (-1, 0, name)
        if name.startswith("model.layers."):
            return (int(name.split(".")[2]), 0, name)
        return (1 << 30, 0 if name.startswith("model.norm") else 1, name)

    def _load(self, name: str, entry: dict[str, Any]):
        """Runs on a loader thread: a verified device tensor for large tensors
        on a CUDA device, else verified host bytes."""
        if self.device.type != "cuda" or int(entry["bytes"]) < DEVICE_MIN_BYTES:
            return _read_verified(self.root, name, entry)
        with torch.cuda.device(self.device):  # loader threads start on device 0
            try:
                st = self._staging.pop()
            except IndexError:
                st = _Staging(self.device, STAGING_CHUNK)
            try:
                return _read_verified_to_device(self.root, name, entry, self.device, st)
            finally:
                self._staging.append(st)

    def _submit(self, name: str) -> None:
        entry = self.manifest["tensors"][name]
        nbytes = int(entry["bytes"])
        self._futures[name] = (self._pool.submit(self._load, name, entry), nbytes)
        self._inflight += nbytes

    def _pump(self) -> None:
        """Keeps reads in flight up to the byte budget (at least one)."""
        while self._next < len(self._order) and (not self._futures or self._inflight < self._budget):
            name = self._order[self._next]
            self._next += 1
            if name not in self._futures and name not in self._taken:
                self._submit(name)

    def _take(self, name: str) -> np.ndarray | torch.Tensor:
        if name not in self._want:
            raise KeyError(name)
        if name not in self._futures:
            self._submit(name)  # out of order, or asked for a second time
        fut, nbytes = self._futures.pop(name)
        self._taken.add(name)
        self._inflight -= nbytes
        try:
            return fut.result()
        finally:
            self._pump()

    def _to_device(self, t: np.ndarray | torch.Tensor) -> torch.Tensor:
        return t if isinstance(t, torch.Tensor) else torch.from_numpy(t).to(self.device)

    def linear(self, module: str) -> tuple[torch.Tensor, torch.Tensor]:
        q = self._to_device(self._take(module + ".weight"))
        s = self._take(module + ".weight_scale")
        s = s.cpu().numpy() if isinstance(s, torch.Tensor) else s
        s32 = s.astype(np.float32)
        if not np.all(np.isfinite(s32)) or np.any(s32 <= 0):
            raise ValueError(f"{module}.weight_scale must be finite and positive")
        return q, torch.from_numpy(s32).to(self.device)

    def dense(self, name: str) -> torch.Tensor:
        return self._to_device(self._take(name)).contiguous()

    def close(self) -> None:
        self._pool.shutdown(wait=True, cancel_futures=True)
        self._futures.clear()
        self._staging.clear()

    def __del__(self):
        pool = getattr(self, "_pool", None)
        if pool is not None:
            pool.shutdown(wait=False, cancel_futures=True)


def write_w8a8_llama_package(directory: str | Path, shape: LlamaShape, weights: Any, *,
                             device: torch.device | str = "cuda",
                             provenance: dict[str, Any] | None = None) -> dict[str, Any]:
    """Quantises (or copies) every Linear of a Llama and writes the
    whole-model package. ``weights`` is a float state dict (quantised on
    ``device`` by the W8A8 kernels) or a weight source with linear()/dense().
    Per-output scales are written as fp16, which holds them exactly (the
    quantiser produces fp16 values); a scale that fp16 does not hold exactly
    is an error."""
    src = as_weight_source(weights, device)
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    entries: dict[str, Any] = {}

    def fname(name: str, dt: np.dtype) -> str:
        return name + (".int8" if dt == _INT8 else ".fp16")

    for mod, n, k in llama_linear_modules(shape):
        q, s = src.linear(mod)
        q = _canonical(q, _INT8, mod + ".weight", dimensions=2)
        s32 = _canonical(s, np.dtype("<f4"), mod + ".weight_scale", dimensions=1)
        if q.shape != (n, k) or s32.shape != (n,):
            raise ValueError(f"{mod}: int8 weight {list(q.shape)} / scales {list(s32.shape)}, want [{n}, {k}] / [{n}]")
        s16 = s32.astype(_FP16)
        if not np.array_equal(s16.astype(np.float32), s32) or np.any(s32 <= 0):
            raise ValueError(f"{mod}.weight_scale is not a positive fp16 value per row")
        entries[mod + ".weight"] = _write_tensor(root, fname(mod + ".weight", _INT8), q)
        entries[mod + ".weight_scale"] = _write_tensor(root, fname(mod + ".weight_scale", _FP16), s16)
    for name, shp in llama_dense_tensors(shape):
        t = _canonical(src.dense(name), _FP16, name, dimensions=len(shp))
        if t.shape != shp:
            raise ValueError(f"{name}: shape {list(t.shape)}, want {list(shp)}")
        entries[name] = _write_tensor(root, fname(name, _FP16), t)
    manifest = {
        "schema_version": SCHEMA_VERSION,
        "package_type": LLAMA_PACKAGE_TYPE,
        "llama_shape": shape.as_dict(),
        "numerical_contract": dict(LLAMA_CONTRACT),
        "tensors": entries,
        "provenance": provenance or {},
    }
    _write_manifest(root, manifest)
    return manifest


def read_llama_package_shape(directory: str | Path) -> LlamaShape:
    """The model geometry recorded in a whole-model package."""
    manifest = _read_manifest(Path(directory))
    if manifest.get("package_type") != LLAMA_PACKAGE_TYPE:
        raise ValueError("not a W8A8 Llama package")
    return _shape_from_manifest(manifest)
