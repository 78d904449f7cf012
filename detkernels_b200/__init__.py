"""detkernels_b200: batch-invariant inference kernels for NVIDIA B200 (sm_100a).

A drop-in for DetKernels' Python API (``kernels.rmsnorm`` / ``kernels.matmul`` /
``kernels.attention`` / ``kernels.tiny_model``, ``gdn``) backed by hand-written
CUDA kernels behind a C ABI (``include/detkernels_b200.h``).
"""
__version__ = "0.1.0"
