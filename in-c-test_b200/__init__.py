"""B200-native MLA hot path of the Kimi-VL low-RAM runtime.

The product is the C-ABI library lib/libkvl_mla_cuda.so (sources in csrc/,
declarations in the repository's include/kvl/).  This package holds its
Python binding (kvl_mla), the multi-GPU host logic (parallel) and the seeded
synthetic-input generator (synth) used by the tests and the benchmark.  The
directory name is not a Python identifier: kvl_pkg.load() at the repository
root imports it under the alias `kvl_b200`.
"""
