"""lmrs_b200 — B200-native (sm_100a) quantized linear layers for lmrs.

AWQ int4 W4A16 and FP8 e4m3 W8A8 linears behind a C-ABI
(``include/lmrs_quant.h``, ``liblmrs_quant.so``) plus the operator layer that
mirrors lmrs's ``LinearOp`` / ``kernels::linear``.  Tensor-parallel sharding of
the quantized projections lives in ``lmrs_b200.tp``.
"""
from .ops import (AwqConfig, DTypeMismatch, LinearConfig, NonContiguous, QuantLinearOp,
                  ShapeMismatch, TensorError, Workspace, awq_dequant, awq_linear, awq_unpack,
                  fp8_linear, fp8_linear_prequant, fp8_quant_rows, quantize_fp8_weight)
from ._lib import LmrsError, load as load_library, read_device_error, set_tuning

__all__ = [
    "AwqConfig", "DTypeMismatch", "LinearConfig", "NonContiguous", "QuantLinearOp",
    "ShapeMismatch", "TensorError", "Workspace", "awq_dequant", "awq_linear", "awq_unpack",
    "fp8_linear", "fp8_linear_prequant", "fp8_quant_rows", "quantize_fp8_weight",
    "LmrsError", "load_library", "read_device_error", "set_tuning",
]
