"""compressai_b200 -- B200-native (sm_100a) VQ2 decode hot path.

Drop-in for the reference ``vq2`` package's decode path: the module names mirror it
(``vq``, ``kernels``, ``runtime``, ``paged_runtime``); compute runs in hand-written CUDA
kernels behind a C-ABI shared library (``include/vq2_b200.h``), loaded with ctypes on first
use. Importing the package does not touch the GPU.
"""
__version__ = "0.1.0"
