"""Checksummed int8 packages on CPU (no compute kernels).

* Linear packages: the fixtures under tests/golden/ref_linear_package_*/ were
  written by the reference's own writer
  (nanopointllm/compression/quantized_tensor_package.py:46-140,
  tests/golden/make_golden.py). nanopointllm_b200.package must load them and,
  given the same tensors, write the same bytes (manifest and tensor files).
  The rejection cases follow tests/test_quantized_tensor_package.py:42-60.
* Whole-model packages: round trip of every tensor through
  write_w8a8_llama_package / PackagedLlamaWeights with oracle-quantised
  weights, and every validation error of the loader.
"""
from __future__ import annotations

import json
import shutil

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden
from oracle import w8a8 as O

REF_PACKAGES = ("ref_linear_package_small", "ref_linear_package_ragged")


def _pkg():
    from nanopointllm_b200 import package
    return package


# ------------------------------------------------------------------ linear packages
@pytest.mark.parametrize("name", REF_PACKAGES)
def test_loads_reference_written_package(name):
    P = _pkg()
    pkg = P.load_quantized_linear_package(GOLDEN / name)
    meta = json.loads((GOLDEN / name / "metadata.json").read_text())
    assert (pkg.m, pkg.n, pkg.k) == (meta["shape"]["m"], meta["shape"]["n"], meta["shape"]["k"])
    assert pkg.activation.dtype == np.int8 and pkg.weight.dtype == np.int8
    assert pkg.weight_scale.dtype == np.float16 and pkg.output_scale is not None
    # the integer golden of the package, through the oracle
    acc = O.int_matmul_nt(pkg.activation, pkg.weight)
    np.testing.assert_array_equal(acc, pkg.activation.astype(np.int64) @ pkg.weight.astype(np.int64).T)


def test_small_package_matches_reference_test_vectors():
    P = _pkg()
    kat = golden("kat.npz")
    pkg = P.load_quantized_linear_package(GOLDEN / "ref_linear_package_small")
    np.testing.assert_array_equal(pkg.activation, kat["pkg_a"])
    np.testing.assert_array_equal(pkg.weight, kat["pkg_w"])
    np.testing.assert_array_equal(O.int_matmul_nt(pkg.activation, pkg.weight), kat["pkg_acc"])
    assert float(pkg.output_scale[0]) == 0.75
    assert pkg.metadata["provenance"] == {"module": "layers.0.self_attn.q_proj"}


@pytest.mark.parametrize("name", REF_PACKAGES)
def test_writer_is_byte_identical_to_reference(tmp_path, name):
    P = _pkg()
    pkg = P.load_quantized_linear_package(GOLDEN / name)
    P.write_quantized_linear_package(
        tmp_path, activation=pkg.activation, weight=pkg.weight, activation_scale=pkg.activation_scale,
        weight_scale=pkg.weight_scale, smooth_scale=pkg.smooth_scale, output_scale=pkg.output_scale,
        bias=pkg.bias, provenance=pkg.metadata["provenance"])
    ref_files = sorted(p.name for p in (GOLDEN / name).iterdir())
    assert sorted(p.name for p in tmp_path.iterdir()) == ref_files
    for f in ref_files:
        assert (tmp_path / f).read_bytes() == (GOLDEN / name / f).read_bytes(), f


def test_linear_package_rejects_corruption(tmp_path):
    P = _pkg()
    shutil.copytree(GOLDEN / "ref_linear_package_small", tmp_path / "p")
    w = tmp_path / "p" / "weight.int8"
    payload = bytearray(w.read_bytes())
    payload[0] ^= 1
    w.write_bytes(payload)
    with pytest.raises(ValueError, match="SHA256 mismatch"):
        P.load_quantized_linear_package(tmp_path / "p")
    w.write_bytes(bytes(payload[:-1]))
    with pytest.raises(ValueError, match="byte count mismatch"):
        P.load_quantized_linear_package(tmp_path / "p")


def test_linear_package_rejects_bad_manifests(tmp_path):
    P = _pkg()
    src = GOLDEN / "ref_linear_package_small"
    for mutate, msg in [
        (lambda m: m.update(schema_version="2.0"), "schema"),
        (lambda m: m["tensors"].pop("smooth_scale"), "missing"),
        (lambda m: m["tensors"]["weight"].update(file="../weight.int8"), "plain file name"),
        (lambda m: m["tensors"]["weight"].update(shape=[4, 3]), "weight shape"),
        (lambda m: m["tensors"]["weight"].update(bytes=13), "size mismatch"),
        (lambda m: m["shape"].update(k=5), "shape"),
    ]:
        d = tmp_path / msg.replace(" ", "_")
        shutil.copytree(src, d)
        meta = json.loads((d / "metadata.json").read_text())
        mutate(meta)
        (d / "metadata.json").write_text(json.dumps(meta))
        with pytest.raises(ValueError, match=msg):
            P.load_quantized_linear_package(d)


def test_linear_package_rejects_incompatible_inputs(tmp_path):
    P = _pkg()
    with pytest.raises(ValueError, match="K dimensions differ"):
        P.write_quantized_linear_package(tmp_path, activation=np.ones((1, 4), np.int8),
                                         weight=np.ones((3, 8), np.int8), activation_scale=1.0,
                                         weight_scale=np.ones(3), smooth_scale=np.ones(8))
    with pytest.raises(ValueError, match="positive"):
        P.write_quantized_linear_package(tmp_path, activation=np.ones((1, 4), np.int8),
                                         weight=np.ones((3, 4), np.int8), activation_scale=1.0,
                                         weight_scale=np.array([1.0, 0.0, 1.0]), smooth_scale=np.ones(4))
    with pytest.raises(ValueError, match="non-finite"):
        P.write_quantized_linear_package(tmp_path, activation=np.ones((1, 4), np.int8),
                                         weight=np.ones((3, 4), np.int8), activation_scale=np.inf,
                                         weight_scale=np.ones(3), smooth_scale=np.ones(4))


# ------------------------------------------------------------ whole-model packages
class _OracleWeights:
    """Weight source of oracle-quantised float weights (CPU tensors)."""

    def __init__(self, sd):
        self.sd = sd
        self.asked = []

    def linear(self, module):
        self.asked.append(module)
        q, s = O.per_output_weight_quant(self.sd[module + ".weight"].float().numpy())
        return torch.from_numpy(q), torch.from_numpy(s.reshape(-1))

    def dense(self, name):
        return self.sd[name]


def _tiny():
    from nanopointllm_b200 import synthetic as S
    shape = S.LlamaShape(hidden=64, heads=2, kv_heads=1, head_dim=32, intermediate=128, layers=2, vocab=100)
    return shape, S.llama_weights(shape, seed=5)


def test_llama_package_round_trip(tmp_path):
    P = _pkg()
    shape, sd = _tiny()
    src = _OracleWeights(sd)
    manifest = P.write_w8a8_llama_package(tmp_path, shape, src, provenance={"weights": "seed 5"})
    assert manifest["package_type"] == P.LLAMA_PACKAGE_TYPE
    assert P.read_llama_package_shape(tmp_path) == shape
    # one int8 weight + fp16 scales per Linear, fp16 embedding / norms
    assert len(manifest["tensors"]) == 2 * (7 * shape.layers + 1) + 2 * shape.layers + 2
    ld = P.PackagedLlamaWeights(tmp_path, "cpu", threads=2, read_ahead_bytes=4096)
    try:
        assert ld.shape == shape
        for mod, n, k in P.llama_linear_modules(shape):
            q, s = ld.linear(mod)
            qr, sr = O.per_output_weight_quant(sd[mod + ".weight"].float().numpy())
            assert q.dtype == torch.int8 and q.shape == (n, k) and s.dtype == torch.float32
            np.testing.assert_array_equal(q.numpy(), qr)
            np.testing.assert_array_equal(s.numpy(), sr.reshape(-1))
        for name, shp in P.llama_dense_tensors(shape):
            t = ld.dense(name)
            assert t.dtype == torch.float16 and tuple(t.shape) == shp
            assert torch.equal(t, sd[name])
        # a second request reads the file again
        assert torch.equal(ld.dense("model.norm.weight"), sd["model.norm.weight"])
        with pytest.raises(KeyError):
            ld.dense("model.layers.9.input_layernorm.weight")
    finally:
        ld.close()


def test_llama_package_read_ahead_is_bounded(tmp_path):
    P = _pkg()
    shape, sd = _tiny()
    P.write_w8a8_llama_package(tmp_path, shape, _OracleWeights(sd))
    biggest = max(int(e["bytes"]) for e in json.loads((tmp_path / "metadata.json").read_text())["tensors"].values())
    ld = P.PackagedLlamaWeights(tmp_path, "cpu", threads=2, read_ahead_bytes=1000)
    try:
        assert ld._inflight <= 1000 + biggest
        for mod, _, _ in P.llama_linear_modules(shape):
            ld.linear(mod)
            assert ld._inflight <= 1000 + biggest
    finally:
        ld.close()


def test_llama_package_detects_corrupt_tensor(tmp_path):
    P = _pkg()
    shape, sd = _tiny()
    P.write_w8a8_llama_package(tmp_path, shape, _OracleWeights(sd))
    f = tmp_path / "model.layers.1.mlp.down_proj.weight.int8"
    payload = bytearray(f.read_bytes())
    payload[17] ^= 0x40
    f.write_bytes(payload)
    ld = P.PackagedLlamaWeights(tmp_path, "cpu")
    try:
        ld.linear("model.layers.0.mlp.down_proj")  # intact tensors still load
        with pytest.raises(ValueError, match="SHA256 mismatch"):
            ld.linear("model.layers.1.mlp.down_proj")
    finally:
        ld.close()


def test_llama_package_rejects_bad_manifests(tmp_path):
    P = _pkg()
    shape, sd = _tiny()
    src = tmp_path / "src"
    P.write_w8a8_llama_package(src, shape, _OracleWeights(sd))
    cases = [
        (lambda m: m.update(package_type=P.LINEAR_PACKAGE_TYPE), "not a W8A8 Llama package"),
        (lambda m: m["tensors"].pop("lm_head.weight_scale"), "missing"),
        (lambda m: m["tensors"].update(extra=dict(m["tensors"]["model.norm.weight"], file="x.fp16")),
         "unexpected"),
        (lambda m: m["llama_shape"].update(hidden=128), "shape"),
        (lambda m: m["llama_shape"].pop("eps"), "llama_shape"),
        (lambda m: m["llama_shape"].update(kv_heads=0), "geometry"),
        (lambda m: m["llama_shape"].update(heads=1, kv_heads=2), "geometry"),
        (lambda m: m["tensors"]["lm_head.weight"].update(dtype="<f2", bytes=2 * 100 * 64), "dtype"),
        (lambda m: m["tensors"]["lm_head.weight"].update(file="/etc/passwd"), "plain file name"),
        (lambda m: m["tensors"]["model.norm.weight"].update(file="lm_head.weight.int8", bytes=128),
         "share one file"),
    ]
    for i, (mutate, msg) in enumerate(cases):
        d = tmp_path / f"case{i}"
        shutil.copytree(src, d)
        meta = json.loads((d / "metadata.json").read_text())
        mutate(meta)
        (d / "metadata.json").write_text(json.dumps(meta))
        with pytest.raises(ValueError, match=msg):
            P.PackagedLlamaWeights(d, "cpu")


def test_llama_package_writer_rejects_inexact_scales(tmp_path):
    P = _pkg()
    shape, sd = _tiny()

    class Off(_OracleWeights):
        def linear(self, module):
            q, s = super().linear(module)
            return q, s * (1 + 2 ** -20)  # not an fp16 value

    with pytest.raises(ValueError, match="fp16"):
        P.write_w8a8_llama_package(tmp_path, shape, Off(sd))
    assert not (tmp_path / "metadata.json").exists()  # no manifest for a failed write
