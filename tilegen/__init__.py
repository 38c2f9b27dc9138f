"""Drop-in alias: ``import tilegen.<module>`` resolves to ``tilegen_b200.<module>``.

Every module of the reference package's public surface is registered under its
reference name, so ``from tilegen.kernels.int8_convrot import _eager_quantize``
and friends return the very same objects as the ``tilegen_b200`` modules (patching
one patches the other).
"""
import importlib
import sys

_MODULES = (
    "kernels", "kernels.hadamard", "kernels.int8_convrot",
    "quant", "quant.weight", "quant.int8_ops", "quant.rowwise",
    "runtime", "runtime.device", "runtime.nvrtc",
    "comfyui", "comfyui.backend", "comfyui.nodes",
)

for _name in _MODULES:
    _mod = importlib.import_module("tilegen_b200." + _name)
    sys.modules[__name__ + "." + _name] = _mod
    _parent, _, _leaf = (__name__ + "." + _name).rpartition(".")
    setattr(sys.modules[_parent], _leaf, _mod)

__version__ = importlib.import_module("tilegen_b200").__version__
