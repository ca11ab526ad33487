"""Shared inputs for the GPU parity tests: identical seeded data on the GPU
(made by libvkcompute's device generators) and on the CPU (made by the
oracle), so every comparison starts from the same bits."""
from __future__ import annotations

import numpy as np
import torch

from oracle import pyoracle as o
from vk_compute_b200 import ops

# Seeds of the reference driver (src/compute.c:18-46).
SEED_X, SEED_GAMMA, SEED_W, SEED_W2 = 4321, 58923, 936, 1348


def host_weight(seed: int, K: int, N: int, bits: int):
    """(data, scale, zero) in the reference's unpacked storage."""
    if bits == 32:
        return o.get_data(seed, K, N), None, None
    if bits == 16:
        return o.get_data_fp16(seed, K, N), None, None
    return o.get_data_quant(seed, K, N, bits)


def device_weight(seed: int, K: int, N: int, bits: int) -> ops.PackedWeight:
    return ops.reference_weight(seed, K, N, bits)


def host_vector(seed: int, n: int) -> np.ndarray:
    return o.get_data(seed, 1, n).ravel()


def device_vector(seed: int, n: int) -> torch.Tensor:
    return ops.reference_vector(seed, n)


def rope_theta(n: int, base: float, head_dim: int) -> np.ndarray:
    p = np.arange(n, dtype=np.float64)
    return (base ** (-2.0 * p / head_dim)).astype(np.float32)
