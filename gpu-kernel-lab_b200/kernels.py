"""Reference-compatible W4A16 decode ops: ``int4_gemv`` and ``int4_lm_head_topk``.

Same names, arguments and ``ValueError`` validation as the reference's
``learning/09_int4/kernels.py:53-99``; the work runs in libkl_b200
(``kl_int4_gemv`` / ``kl_int4_lm_head_topk``) instead of Triton.  Results are
in the activation dtype (f32 accumulation, one rounding), and the head's
top-1 ties resolve to the lowest vocabulary index.
"""
from __future__ import annotations

import torch

from . import ops as _ops  # noqa: F401  (registers torch.ops.kl_b200)
from .quantization import PackedInt4


def _validate(x, packed, block_n):
    packed.validate()
    if not x.is_cuda or x.device != packed.data.device:
        raise ValueError('activation and packed weights must be on one CUDA device')
    if x.ndim != 1 or x.numel() != packed.shape[1] or not x.is_contiguous():
        raise ValueError('one contiguous decode token x[K] required')
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError('activations must be FP16 or BF16')
    if block_n not in (8, 16, 32, 64):
        raise ValueError('block_n must be 8,16,32,64')
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError('inference only')


def int4_gemv(x, packed: PackedInt4, block_n=32):
    _validate(x, packed, block_n)
    return torch.ops.kl_b200.int4_gemv(x, packed.data, packed.scales, packed.group_size, block_n)


def int4_lm_head_topk(x, packed: PackedInt4, top_k=1, block_n=32):
    """Fused lm_head projection + selection; returns (values f32 [top_k], ids int64 [top_k]).

    Does not produce full logits; ties for top-1 select the lowest vocabulary
    index.  Caller must supply finite inputs.
    """
    _validate(x, packed, block_n)
    n, k = packed.shape
    if not 1 <= top_k <= min(8, block_n, n):
        raise ValueError('top_k must be between 1 and min(8,block_n,vocabulary)')
    return torch.ops.kl_b200.int4_lm_head_topk(x, packed.data, packed.scales, packed.group_size, top_k, block_n)
