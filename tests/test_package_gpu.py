"""Checksummed int8 packages on the GPU.

* integer_golden of the reference-written linear packages through the
  tcgen05 linear's int32 accumulator output, against the oracle and the
  reference test's golden (tests/test_quantized_tensor_package.py:26-39);
* a whole-model package written from float weights (quantised by
  npl_quant_rows) holds exactly the oracle's int8 weights and scales;
* a runner built from the package (W8A8LlamaRunner.from_package) generates
  the same tokens and bit-identical logits as one built from the float
  weights, eager and under the decode CUDA graph.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden
from oracle import w8a8 as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["ref_linear_package_small", "ref_linear_package_ragged"])
def test_integer_golden_on_gpu(name):
    from nanopointllm_b200 import package as P
    pkg = P.load_quantized_linear_package(GOLDEN / name)
    acc = pkg.integer_golden("cuda:0")
    np.testing.assert_array_equal(acc, O.int_matmul_nt(pkg.activation, pkg.weight))
    if name.endswith("small"):
        np.testing.assert_array_equal(acc, golden("kat.npz")["pkg_acc"])


def test_package_from_float_weights_matches_oracle(tmp_path):
    from nanopointllm_b200 import package as P, synthetic as S
    shape = S.TINY
    sd = S.llama_weights(shape, seed=0)
    P.write_w8a8_llama_package(tmp_path, shape, sd, device="cuda:0")
    ld = P.PackagedLlamaWeights(tmp_path, "cpu")
    try:
        for mod, _, _ in P.llama_linear_modules(shape):
            q, s = ld.linear(mod)
            qr, sr = O.per_output_weight_quant(sd[mod + ".weight"].float().numpy())
            np.testing.assert_array_equal(q.numpy(), qr, err_msg=mod)
            np.testing.assert_array_equal(s.numpy(), sr.reshape(-1), err_msg=mod)
    finally:
        ld.close()


def test_runner_from_package_is_bit_identical(tmp_path):
    from test_runner_gpu import _generate
    from nanopointllm_b200 import package as P, runner as R, synthetic as S
    dev = torch.device("cuda:0")
    shape = S.TINY
    sd = S.llama_weights(shape, seed=0)
    lengths = [37, 5, 64, 19]
    prompts = S.decode_prompts(len(lengths), shape.vocab, lengths, seed=2)
    bs, per_seq = 16, 6
    nb = len(lengths) * per_seq
    bt = S.permuted_block_tables(len(lengths), per_seq, nb, seed=3).numpy()
    full = R.W8A8LlamaRunner(shape, sd, device=dev, num_blocks=nb, block_size=bs)
    t_ref, l_ref = _generate(full, prompts, bt, 5, dev)
    del full
    P.write_w8a8_llama_package(tmp_path, shape, sd, device=dev, provenance={"weights": "synthetic seed 0"})
    for graph in (False, True):
        run = R.W8A8LlamaRunner.from_package(tmp_path, device=dev, num_blocks=nb, block_size=bs)
        assert run.shape == shape
        t, lg = _generate(run, prompts, bt, 5, dev, graph=graph)
        np.testing.assert_array_equal(t, t_ref)
        np.testing.assert_array_equal(lg, l_ref)
        del run
    # a corrupt tensor stops the build before a runner exists
    f = tmp_path / "model.layers.1.self_attn.o_proj.weight.int8"
    payload = bytearray(f.read_bytes())
    payload[123] ^= 1
    f.write_bytes(payload)
    with pytest.raises(ValueError, match="SHA256 mismatch"):
        R.W8A8LlamaRunner.from_package(tmp_path, device=dev, num_blocks=nb, block_size=bs)
