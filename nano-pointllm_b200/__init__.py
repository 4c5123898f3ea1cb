"""nanopointllm_b200: B200-native (sm_100a) W8A8 linear + paged-decode path.

The directory is named ``nano-pointllm_b200`` and is imported under the module
name ``nanopointllm_b200`` (the entry points register it with importlib).

Public surface, mirroring the reference ``nanopointllm`` API for this path:

* ``nanopointllm_b200.w8a8``            - the W8A8 contract on the GPU under
  the reference's names and signatures (quantize_symmetric,
  scale_from_absmax, per_output_weight_qdq, static_activation_scale,
  static_activation_qdq, dynamic_per_token_activation_qdq,
  integer_linear_per_output_reference), plus the decode-path forms
  (per_output_weight_quant, dynamic_per_token_quant, linear_q, W8A8Linear)
* ``nanopointllm_b200.paged_attention`` - store_kvcache, paged_decode_attention,
  rope_store_kvcache
* ``nanopointllm_b200.runner``          - W8A8 Llama decode runner
  (inject/quantize a model, prefill + decode steps, CUDA-graph decode)
* ``nanopointllm_b200.tp``              - the same runner split over GPUs
  (tensor parallel: column-parallel QKV / gate-up / LM head, row-parallel
  O / down with int32 all-reduce)
* ``nanopointllm_b200.serving``         - continuous-batching driver (block
  manager, FIFO two-queue scheduler, mixed prefill/decode steps, per-bucket
  decode graphs) and the data-parallel request router across replicas
* ``nanopointllm_b200.package``         - checksummed int8 packages: the
  reference's single-linear package schema and a whole-model package the
  runners start from without re-quantising (``W8A8LlamaRunner.from_package``)

Every compute call goes through the C-ABI library ``libnpl_w8a8.so`` built
from ``csrc/``; there is no CPU or library fallback.
"""
from __future__ import annotations

__all__ = ["w8a8", "paged_attention", "runner", "synthetic", "tp", "package", "serving"]
