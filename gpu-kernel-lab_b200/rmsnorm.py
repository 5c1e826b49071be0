"""Qwen RMSNorm and the fused residual-add + RMSNorm on the B200 kernels.

Mirrors ``learning/03_rmsnorm/qwen_rmsnorm.py:66-131`` of the reference:
* the same two calls and return values: ``y``, or ``(y, residual_stream)``;
* the same argument checks, each raising ``ValueError`` with the same wording;
* the same operation order: the normalised value is rounded to the input dtype
  before the weight multiply, as Qwen3RMSNorm does.

``num_warps`` is checked as the reference checks it and is otherwise only a
hint: the kernel sizes its own launch. The reference's Triton names
(``triton_qwen_rmsnorm``, ``triton_qwen_residual_rmsnorm``) are kept as aliases
so that callers can swap the import. The reference's decode runtime calls the
residual form before each layer's QKV and gate_up projection
(``learning/12_decode_runtime/decode_runtime.py:72,90``).

Widths up to ``KL_RMSNORM_MAX_N`` (16384) are accepted; the reference's kernel
stops at 4096.
"""
from __future__ import annotations

import math

import torch

from . import _native as N

MAX_N = 16384


def _check_common(x, weight, epsilon, num_warps, precise_math, extra_grad=()):
    if x.ndim < 1 or x.shape[-1] == 0:
        raise ValueError('input must have a nonempty last dimension')
    if not x.is_cuda or weight.device != x.device:
        raise ValueError('input and weight must be on the same CUDA device')
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16) or weight.dtype != x.dtype:
        raise ValueError('input and weight must have matching FP32/FP16/BF16 dtype')
    if weight.ndim != 1 or weight.numel() != x.shape[-1]:
        raise ValueError('weight must be a vector matching the last dimension')
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError('contiguous input and weight required')
    if not math.isfinite(epsilon) or epsilon <= 0:
        raise ValueError('epsilon must be finite and positive')
    if num_warps not in (2, 4, 8):
        raise ValueError('num_warps must be 2, 4, or 8')
    if not isinstance(precise_math, bool):
        raise ValueError('precise_math must be bool')
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, weight, *extra_grad)):
        raise ValueError('inference only; use torch.inference_mode()')
    if x.shape[-1] > MAX_N:
        raise ValueError(f'widths up to {MAX_N} are supported')


def _launch(x, residual, weight, epsilon, precise_math, y, residual_out):
    n = x.shape[-1]
    rows = x.numel() // n
    if rows == 0:
        return
    with torch.cuda.device(x.device):
        N.check(N.lib().kl_rmsnorm(N.ptr(x), N.ptr(residual), N.ptr(weight), N.act_dtype_code(x.dtype), rows, n,
                                   float(epsilon), int(precise_math), N.ptr(y), N.ptr(residual_out),
                                   N.stream_handle(x.device)))


def qwen_rmsnorm(x, weight, epsilon=1e-6, num_warps=4, precise_math=False):
    """``weight * T(x * rsqrt(mean(x^2) + eps))`` per row, in ``x``'s dtype."""
    _check_common(x, weight, epsilon, num_warps, precise_math)
    output = torch.empty_like(x)
    _launch(x, None, weight, epsilon, precise_math, output, None)
    return output


def qwen_residual_rmsnorm(x, residual, weight, epsilon=1e-6, num_warps=4, precise_math=False):
    """Return ``(normalized, residual_stream)`` where ``residual_stream = x + residual``
    (rounded to the dtype, as a standalone add would store it) and ``normalized``
    is its Qwen RMSNorm; one pass over memory."""
    if residual.shape != x.shape or residual.dtype != x.dtype or residual.device != x.device:
        raise ValueError('residual must match input shape, dtype, and device')
    if not residual.is_contiguous():
        raise ValueError('contiguous residual required')
    _check_common(x, weight, epsilon, num_warps, precise_math, extra_grad=(residual,))
    output, residual_output = torch.empty_like(x), torch.empty_like(x)
    _launch(x, residual, weight, epsilon, precise_math, output, residual_output)
    return output, residual_output


# the reference's names, for callers that swap the import
triton_qwen_rmsnorm = qwen_rmsnorm
triton_qwen_residual_rmsnorm = qwen_residual_rmsnorm
