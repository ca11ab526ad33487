"""vk_compute_b200: vk-compute's matrix-vector decode path (GEMV, fused
RmsNorm-GEMV / -Rope / SwiGLU, decode attention, prefill GEMM) as sm_100a
CUDA kernels behind the reference's C ABI.

The compiled library is libvkcompute.so in this directory (build with
``python -m vk_compute_b200._build``); ``ops`` wraps its native entry points
for torch tensors and ``dropin`` exposes the reference's session / buffer /
execute ABI.
"""
from ._lib import LIB_PATH, VkcError, lib

__all__ = ["LIB_PATH", "VkcError", "lib"]
