"""Benchmarks beyond the headline ``bench.py``: the collective sweep (``collective_sweep``) and the
decode-kernel microbenchmark (``decode_kernels``)."""
