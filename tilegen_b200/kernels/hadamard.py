"""Group-Hadamard helpers (API of tilegen/kernels/hadamard.py).

The ConvRot rotation of a group of G = 4^n elements is the n-fold Kronecker
power of the 4x4 core below, scaled by 1/sqrt(G).  The core has its -1 entries
on the anti-diagonal (tilegen/kernels/hadamard.py:15), so entry (i, j) of the
G x G matrix is -1 to the number of base-4 digit positions d where
j_d == 3 - i_d (i.e. j_d == i_d XOR 3), divided by sqrt(G) = 2^n, which is
exact in every float dtype.
"""
from __future__ import annotations

import functools

import torch

_H4 = [[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]]


def _validate_group_size(group_size: int) -> None:
    """Powers of four only, as tilegen/kernels/hadamard.py:18-22."""
    if group_size < 4 or (group_size & (group_size - 1)) != 0:
        raise ValueError(f"group_size must be a power of two >= 4, got {group_size}")
    if (group_size.bit_length() - 1) % 2:
        raise ValueError(f"group_size must be a power of 4, got {group_size}")


def _digits(size: int) -> int:
    return (size.bit_length() - 1) // 2


@functools.lru_cache(maxsize=16)
def _hadamard(device_type: str, device_index: int, dtype: torch.dtype, size: int) -> torch.Tensor:
    """Cached normalised Hadamard matrix of order ``size`` (a power of 4)."""
    _validate_group_size(size)
    device = torch.device(device_type, device_index) if device_type == "cuda" else torch.device(device_type)
    n = _digits(size)
    idx = torch.arange(size)
    flips = torch.zeros(size, size, dtype=torch.int64)
    for d in range(n):
        di = (idx >> (2 * d)) & 3
        flips += (di[None, :] == (di[:, None] ^ 3)).to(torch.int64)
    sign = 1.0 - 2.0 * (flips % 2).to(torch.float64)
    return (sign * (2.0 ** -n)).to(device=device, dtype=dtype)


def build_hadamard(size: int, device, dtype: torch.dtype) -> torch.Tensor:
    """Normalised Hadamard matrix of order ``size`` (4, 16, 64, 256, ...)."""
    if isinstance(device, torch.device):
        device_type, device_index = device.type, device.index or 0
    else:
        device_type, device_index = str(device), 0
    return _hadamard(device_type, device_index, dtype, size)


def rotate_by_group(x: torch.Tensor, h: torch.Tensor, group_size: int) -> torch.Tensor:
    """Rotate ``x [*, K]`` group-wise: ``x.reshape(*, K/G, G) @ h``."""
    lead, k = x.shape[:-1], x.shape[-1]
    if k % group_size:
        raise ValueError(f"K={k} must be divisible by group_size={group_size}")
    y = torch.matmul(x.reshape(*lead, k // group_size, group_size), h.to(x.dtype))
    return y.reshape(*lead, k)
