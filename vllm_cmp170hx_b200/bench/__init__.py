"""Micro-benchmarks of the hot kernels at the BASELINE shapes (``python -m vllm_cmp170hx_b200.bench.kernels``)."""
