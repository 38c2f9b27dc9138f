"""tilegen_b200: the int8_convrot hot path of tilegen, rebuilt for B200 (sm_100a).

* ``tilegen_b200.kernels`` / ``.quant`` / ``.comfyui`` / ``.runtime`` keep the
  reference package's API (the top-level ``tilegen`` package re-exports them
  under the reference's module names, so existing imports keep working).
* ``tilegen_b200.ops`` are the torch wrappers of the C ABI
  (``include/tilegen_b200.h``), also registered as ``torch.ops.tilegen.*``.
* ``tilegen_b200.sharding`` row-shards the path across GPUs.

Importing the package does not load the CUDA library; the first op does, and
raises if it is missing (there is no fallback implementation).
"""
__version__ = "0.1.0"
