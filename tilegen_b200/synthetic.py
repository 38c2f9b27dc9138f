"""Seeded synthetic inputs for the int8_convrot workloads.

No public dataset is involved: the workloads are DiT projection layers fed with
activations that have a few large "outlier" channels, which is the case the
group-Hadamard rotation exists for.  Recipe (one ``torch.Generator`` per tensor,
generated on the CPU in fp32, then cast and moved):

* activations ``x[M, K] ~ N(0, 1)``; for the FFN-down projection they are first
  passed through the erf GELU.  Outlier channels: ``idx = randperm(K)[:round(p*K)]``
  and ``x[:, idx] *= s`` (p=1 %, s=30; FFN-down p=0.5 %, s=50).
* weights ``W[N, K] ~ N(0, 0.02)``.
* for the normalisation fused in front of a projection: a residual stream
  (per-channel offsets, 0.5 % of channels x20) and adaLN modulation vectors
  ``N(0, 0.1)`` (``residual_stream``, ``dit_modulation``).

``device="cuda"`` generates on the GPU instead (same distribution, different
stream of numbers), which the benchmark uses for the large shapes.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

# (name, K, N) of one 14B-class video DiT block (hidden 5120, FFN 13824).
DIT_SHAPES = (
    ("qkv_proj", 5120, 15360),
    ("o_proj", 5120, 5120),
    ("ffn_up", 5120, 13824),
    ("ffn_down", 13824, 5120),
)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def outlier_activations(
    m: int,
    k: int,
    *,
    seed: int = 0,
    frac: float = 0.01,
    scale: float = 30.0,
    gelu: bool = False,
    dtype: torch.dtype = torch.float16,
    device="cpu",
) -> torch.Tensor:
    """``x[m, k]``: N(0,1) (optionally GELU'd) with ``round(frac*k)`` channels scaled."""
    dev = torch.device(device)
    x = torch.randn(m, k, generator=_gen(seed, dev), device=dev, dtype=torch.float32)
    if gelu:
        x = F.gelu(x)
    n_out = int(round(frac * k))
    if n_out:
        idx = torch.randperm(k, generator=_gen(seed, dev), device=dev)[:n_out]
        x[:, idx] *= scale
    return x.to(dtype)


def dit_activations(name: str, m: int, *, seed: int = 0, dtype=torch.float16, device="cpu"):
    """Activations for one DiT projection: FFN-down gets GELU inputs, 0.5 % x50."""
    k = dict((s[0], s[1]) for s in DIT_SHAPES)[name]
    if name == "ffn_down":
        return outlier_activations(m, k, seed=seed, frac=0.005, scale=50.0, gelu=True,
                                   dtype=dtype, device=device)
    return outlier_activations(m, k, seed=seed, dtype=dtype, device=device)


def gaussian_weight(n: int, k: int, *, seed: int = 0, std: float = 0.02,
                    dtype=torch.float32, device="cpu") -> torch.Tensor:
    """``W[n, k] ~ N(0, std)``."""
    dev = torch.device(device)
    w = torch.randn(n, k, generator=_gen(seed, dev), device=dev, dtype=torch.float32) * std
    return w.to(dtype)


def residual_stream(m: int, k: int, *, seed: int = 0, dtype=torch.float16, device="cpu") -> torch.Tensor:
    """A DiT block's residual stream ``h[m, k]`` (the input of its LayerNorm): per-channel
    offsets ``N(0, 0.5)`` plus ``N(0, 1)`` noise, with 0.5 % of the channels x20 (the
    large "massive activation" channels such streams carry)."""
    dev = torch.device(device)
    g = _gen(seed, dev)
    offset = torch.randn(k, generator=g, device=dev) * 0.5
    h = torch.randn(m, k, generator=g, device=dev) + offset
    idx = torch.randperm(k, generator=g, device=dev)[: max(1, round(0.005 * k))]
    h[:, idx] *= 20.0
    return h.to(dtype)


def dit_modulation(vectors: int, k: int, *, seed: int = 0, dtype=torch.float16, device="cpu"):
    """``(scale, shift)``, each ``[vectors, k] ~ N(0, 0.1)``: the adaLN modulation a DiT
    block applies after its LayerNorm, one vector per sample."""
    dev = torch.device(device)
    g = _gen(seed, dev)
    scale = torch.randn(vectors, k, generator=g, device=dev) * 0.1
    shift = torch.randn(vectors, k, generator=g, device=dev) * 0.1
    return scale.to(dtype), shift.to(dtype)
