"""Helpers shared by the tests."""
from __future__ import annotations

import numpy as np
import torch

DT_NAME = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}


def raw16(t: torch.Tensor) -> np.ndarray:
    """fp16/bf16 tensor -> numpy uint16 bit patterns (CPU copy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def oracle_input(x: torch.Tensor) -> np.ndarray:
    x = x.detach().cpu().contiguous()
    return x.numpy() if x.dtype == torch.float32 else raw16(x)


def out_bits(y: torch.Tensor) -> np.ndarray:
    """Output tensor -> numpy array comparable with the oracle's output."""
    y = y.detach().cpu().contiguous()
    return y.numpy() if y.dtype == torch.float32 else raw16(y)


def rel_fro(a, b) -> float:
    a = torch.as_tensor(a).double()
    b = torch.as_tensor(b).double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
