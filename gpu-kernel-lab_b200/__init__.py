"""B200-native (sm_100a) weight-only quantized linear layer (W8A16 / W4A16).

A drop-in for the quantized-Linear path of yashlabs-trying/gpu-kernel-lab:
the reference's Python interfaces (``project``, ``quantize_int8``,
``dequantize_int8``, ``CalibratedInt8``, ``PackedInt4``, ``quantize_int4``,
``dequantize_int4``, ``int4_gemv``, ``int4_lm_head_topk``, the
``serving/kernel_policy.py`` dispatch contract) backed by hand-written CUDA
kernels in ``libkl_b200.so`` (C ABI: ``include/kl_b200.h``).

The directory name contains hyphens, so import it with
``importlib.import_module("gpu-kernel-lab_b200")``.
"""
from . import _native, kernel_policy, ops, sharded_head
from .activation_int8 import (CalibratedInt8, RowwiseInt8, dequantize_int8, dequantize_int8_rowwise,
                              quantize_int8, quantize_int8_rowwise)
from .cuda_decode import extension, project
from .kernels import int4_gemv, int4_lm_head_topk
from .linear import GroupedLinear, QuantLinear, lm_head_topk, quant_linear, weight_spec
from .quantization import (PackedInt4, PackedInt4Asym, dequantize_int4, dequantize_int4_asym, quantize_int4,
                           quantize_int4_asym)
from .native_ops import dequantize_native
from .adapters import install_quantized_executor, install_quantized_projections
from .quant_tensor import QuantWeight
from .packed_store import export_packed, install_packed, load_packed, save_packed
from .rmsnorm import qwen_residual_rmsnorm, qwen_rmsnorm
from .sharded_head import VocabShardedHead
from .kernel_policy import QwenKernelPolicy, load_qwen_policy, select_qwen_policy

__all__ = [
    "CalibratedInt8", "RowwiseInt8", "PackedInt4", "PackedInt4Asym", "QuantLinear",
    "quantize_int8", "dequantize_int8", "quantize_int8_rowwise", "dequantize_int8_rowwise",
    "quantize_int4", "dequantize_int4", "quantize_int4_asym", "dequantize_int4_asym",
    "project", "extension", "int4_gemv", "int4_lm_head_topk", "quant_linear", "lm_head_topk", "weight_spec", "GroupedLinear",
    "dequantize_native", "install_quantized_projections", "kernel_policy", "QwenKernelPolicy", "load_qwen_policy",
    "select_qwen_policy", "sharded_head", "VocabShardedHead",
    "export_packed", "save_packed", "load_packed", "install_packed", "packed_store",
    "qwen_rmsnorm", "qwen_residual_rmsnorm", "rmsnorm", "ops", "QuantWeight", "install_quantized_executor",
]
