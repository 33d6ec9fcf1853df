"""lmc_b200 - B200-native quantized-weight hot path for LMc.

The product is the CUDA/C shared library lmc_b200/liblmc_b200.so (C-ABI in
include/lmc_cuda.h).  This package holds its Python bindings (`runtime`) and
the seeded synthetic GGUF generator (`synth`) used by tests and the bench.
"""
