"""CPU oracle for the W8A8 linear + paged-decode path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the reference
algorithms of nanopointllm (compression/w8a8.py, llama/lightweight_runner.py,
llama/paged_attention.py and the HF Llama RoPE they call). It is the checker
for the CUDA kernels: only tests/, __graft_entry__.smoke() and the CPU-baseline
leg of bench.py may import it. The product path never calls it, and there is no
CPU fallback built on it.

Parity pins: the restatement is checked against the reference's own
known-answer vectors and against fixtures produced by importing the reference
(tests/golden/make_golden.py -> tests/golden/*.npz).
"""
