"""Reference-compatible decode projection: ``project(x, weight, ...)``.

Same call shape as the reference's ``learning/10_cuda_decode/cuda_decode.py:17-25``
(and its C++ op ``warp_gemv.cu:56-90``): ``x`` is one bf16 decode token ``[K]``,
``weight`` is a bf16 ``[N,K]`` tensor, a ``CalibratedInt8``-like object, or (new)
a ``RowwiseInt8``; with ``swiglu=True`` gate rows precede up rows and the
result is ``bf16(silu(bf16 gate)) * bf16(up)`` of length N/2.  Precondition
failures raise ``RuntimeError`` as the reference's ``TORCH_CHECK`` does;
``warps``/``persistent`` are validated and accepted for compatibility (the B200
launch geometry is chosen by the library).
"""
from __future__ import annotations

import torch

from . import _native as N
from . import ops as _ops  # noqa: F401  (registers torch.ops.kl_b200)
from .activation_int8 import RowwiseInt8
from .linear import quant_linear


def extension():
    """The loaded native library (the reference JIT-builds its extension here)."""
    return N.lib()


def project(x, weight, *, warps=4, persistent=False, swiglu=False):
    """weight is BF16 [N,K], CalibratedInt8 or RowwiseInt8; gate rows precede up rows."""
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError('inference only')
    w = weight if isinstance(weight, torch.Tensor) else weight.data
    if not (x.is_cuda and w.is_cuda and x.device == w.device):
        raise RuntimeError("same CUDA device required")
    if x.dtype != torch.bfloat16 or x.dim() != 1 or not x.is_contiguous():
        raise RuntimeError("x: contiguous BF16 vector")
    if w.dim() != 2 or not w.is_contiguous() or w.shape[0] == 0 or w.shape[1] == 0 or w.shape[1] != x.numel():
        raise RuntimeError("w: contiguous nonempty [N,K]")
    if warps not in (1, 4, 8):
        raise RuntimeError("warps must be 1,4,8")
    if swiglu and w.shape[0] % 2:
        raise RuntimeError("gate/up requires two equal row sets")
    if isinstance(weight, RowwiseInt8):
        return quant_linear(x, weight, swiglu=swiglu)
    n, k = w.shape
    if isinstance(weight, torch.Tensor):
        if w.dtype != torch.bfloat16:
            raise RuntimeError("BF16 or INT8 weights required")
        return torch.ops.kl_b200.project(x, w, None, None, 128, warps, bool(persistent), bool(swiglu))
    if weight.scales.dtype != torch.float32 or weight.inverse.dtype != torch.float32 or \
            not weight.scales.is_contiguous() or not weight.inverse.is_contiguous():
        raise RuntimeError("FP32 contiguous scaling buffers required")
    if weight.scales.device != x.device or weight.inverse.device != x.device:
        raise RuntimeError("scales must share device")
    g = int(weight.group_size)
    if g <= 0 or k % g or weight.scales.shape != (n, k // g) or weight.inverse.shape != (k,):
        raise RuntimeError("scaling shapes incorrect")
    return torch.ops.kl_b200.project(x, w, weight.scales, weight.inverse, g, warps, bool(persistent), bool(swiglu))
