"""Inference side products: 4-bit weight quantisation (round-to-nearest and GPTQ), the W4A16 layer with its sm_100a
kernels and C++ CPU reference, an efficiency-benchmark predictor wrapper and an MMLU scorer."""
from .quantize import gptq_quantize_weight, quantize_linear, quantize_model
from .w4a16 import QuantLinear, pack_int4, unpack_int4

__all__ = ["QuantLinear", "pack_int4", "unpack_int4", "gptq_quantize_weight", "quantize_linear", "quantize_model"]
from .wna16 import BitsLinear, pack_bits, quantize_groups_bits, unpack_bits  # noqa: F401,E402
