"""ConvRot kernels (API of tilegen/kernels): rotate+quant on sm_100a."""
from .hadamard import build_hadamard
from .int8_convrot import quantize_convrot, quantize_convrot_fht

__all__ = ["build_hadamard", "quantize_convrot", "quantize_convrot_fht"]
