"""Weight-side ConvRot quantisation and the fused INT8 GEMM + dequant (API of tilegen/quant)."""
from .int8_ops import int8_matmul_dequant_chunked
from .rowwise import quantize_rowwise
from .weight import quantize_convrot_weight

__all__ = ["int8_matmul_dequant_chunked", "quantize_convrot_weight", "quantize_rowwise"]
