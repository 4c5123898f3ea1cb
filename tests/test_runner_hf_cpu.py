"""Host-side mapping of an HF LlamaForCausalLM onto the W8A8 runner (no GPU):
the geometry read from the HF config, and the state-dict names the runner
consumes, which must be exactly the model's own."""
from __future__ import annotations

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _cfg(**kw):
    base = dict(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                num_key_value_heads=4, head_dim=128, vocab_size=1000, max_position_embeddings=512,
                rms_norm_eps=1e-6, tie_word_embeddings=False, rope_theta=10000.0)
    base.update(kw)
    return transformers.LlamaConfig(**base)


def test_shape_from_hf_config_7b_and_tiny():
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    seven = _cfg(hidden_size=4096, intermediate_size=11008, num_hidden_layers=32, num_attention_heads=32,
                 num_key_value_heads=32, head_dim=None, vocab_size=32003, max_position_embeddings=2048)
    assert R.shape_from_hf_config(seven) == S.LLAMA_7B
    assert R.shape_from_hf_config(_cfg()) == S.TINY
    gqa = R.shape_from_hf_config(_cfg(num_key_value_heads=2, rope_theta=5e5, rms_norm_eps=1e-5))
    assert (gqa.kv_heads, gqa.rope_theta, gqa.eps) == (2, 5e5, 1e-5)


def test_runner_consumes_exactly_the_hf_state_dict_names():
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    with torch.device("meta"):
        model = transformers.LlamaForCausalLM(_cfg())
    shape = R.shape_from_hf_config(model.config)
    hf = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    ours = {name: shp for name, shp, _ in S.llama_weight_names(shape)}
    assert hf == ours
