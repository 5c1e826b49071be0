"""Thin wrappers over native entry points that are not GEMMs."""
from __future__ import annotations

import torch

from . import _native as N


def dequantize_native(weight) -> torch.Tensor:
    """f32 ``[N, K]`` dequantised weights computed on the GPU by ``kl_dequantize``
    with the arithmetic the GEMM kernels use (bit-exact vs. the reference
    dequantisers)."""
    from .linear import weight_spec
    fmt, data, scales, zeros, inverse, n, k, group = weight_spec(weight)
    if not data.is_cuda:
        raise RuntimeError("dequantize_native needs CUDA tensors")
    out = torch.empty((n, k), dtype=torch.float32, device=data.device)
    with torch.cuda.device(data.device):
        N.check(N.lib().kl_dequantize(N.ptr(data), fmt, n, k, group, N.ptr(scales), N.ptr(zeros), N.ptr(inverse),
                                      N.ptr(out), N.stream_handle(data.device)))
    return out
