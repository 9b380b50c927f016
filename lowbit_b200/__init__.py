"""lowbit_b200: lowbit's fused dequantize + GEMM kernels, rebuilt for NVIDIA B200 (sm_100a).

Drop-in for the hot path of lowbit (src/lowbit/__init__.py): the same packed
formats and quantizers, and GEMMs with the same names and arguments, running
as hand-written CUDA kernels behind a C ABI (include/lowbit_b200.h).
"""
from .formats import (GROUP, MXBLOCK, AMXInt4Weights, Int4Weights, Int8Acts, MXFP4Weights, pack_amx,
                      quantize_act_int8, quantize_int4, quantize_mxfp4)
from .kernels import (Params, amx_available, cpu_info, gemm_mxfp4, gemm_w4a8, gemm_w4a8_amx, gemm_w4a16,
                      gpu_info, w4a8_group_acc_amx)

__version__ = "0.1.0"
__all__ = [
    "GROUP", "MXBLOCK", "AMXInt4Weights", "Int4Weights", "Int8Acts", "MXFP4Weights", "Params", "amx_available",
    "cpu_info", "gemm_mxfp4", "gemm_w4a8", "gemm_w4a8_amx", "gemm_w4a16", "gpu_info", "pack_amx",
    "quantize_act_int8", "quantize_int4", "quantize_mxfp4", "w4a8_group_acc_amx",
]
