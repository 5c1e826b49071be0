"""W4A16 weight containers and quantisers.

Mirrors the reference's ``learning/09_int4/quantization.py`` (``PackedInt4``,
``quantize_int4``, ``dequantize_int4``: symmetric absmax/7 codes, f32 group
scales, low nibble = even k) and adds the asymmetric format of BASELINE.json
config 3 (``PackedInt4Asym``: unsigned codes, bf16 scale and bf16 zero point
per group, ``w = (q - z) * s``).

CUDA weights are packed by the native kernel (``kl_quantize_w4``); CPU weights
by the same arithmetic in torch (quantisation is offline).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N


@dataclass(frozen=True)
class PackedInt4:
    """Reference format (``quantization.py:7-32``)."""
    data: torch.Tensor       # uint8 [N, K/2], low nibble precedes high nibble
    scales: torch.Tensor     # f32 [N, K/group_size]
    group_size: int

    @property
    def shape(self):
        return (self.data.shape[0], self.data.shape[1] * 2)

    @property
    def storage_bytes(self):
        return self.data.numel() + self.scales.numel() * 4

    def validate(self):
        if self.group_size not in (32, 64, 128):
            raise ValueError('group_size must be 32, 64, or 128')
        if self.data.ndim != 2 or self.data.dtype != torch.uint8:
            raise ValueError('packed data must be uint8 [N,K/2]')
        n, k = self.shape
        if n == 0 or k == 0 or k % self.group_size:
            raise ValueError('positive dimensions and K divisible by group_size required')
        if self.scales.shape != (n, k // self.group_size) or self.scales.dtype != torch.float32:
            raise ValueError('scales must be FP32 [N,K/group_size]')
        if self.data.device != self.scales.device or not self.data.is_contiguous() or not self.scales.is_contiguous():
            raise ValueError('contiguous colocated buffers required')


@dataclass(frozen=True)
class PackedInt4Asym:
    """BASELINE config 3 format: unsigned nibbles, bf16 scales / zeros per group."""
    data: torch.Tensor       # uint8 [N, K/2]
    scales: torch.Tensor     # bf16 [N, K/group_size]
    zeros: torch.Tensor      # bf16 [N, K/group_size] (integers 0..15)
    group_size: int

    @property
    def shape(self):
        return (self.data.shape[0], self.data.shape[1] * 2)

    @property
    def storage_bytes(self):
        return self.data.numel() + 2 * (self.scales.numel() + self.zeros.numel())

    def validate(self):
        if self.group_size <= 0 or self.group_size % 2:
            raise ValueError('group_size must be positive and even')
        if self.data.ndim != 2 or self.data.dtype != torch.uint8:
            raise ValueError('packed data must be uint8 [N,K/2]')
        n, k = self.shape
        if n == 0 or k == 0 or k % self.group_size:
            raise ValueError('positive dimensions and K divisible by group_size required')
        for name, t in (('scales', self.scales), ('zeros', self.zeros)):
            if t.shape != (n, k // self.group_size) or t.dtype != torch.bfloat16:
                raise ValueError(f'{name} must be BF16 [N,K/group_size]')
            if t.device != self.data.device or not t.is_contiguous():
                raise ValueError('contiguous colocated buffers required')
        if not self.data.is_contiguous():
            raise ValueError('contiguous colocated buffers required')


def _check_weight(weight, group_size, groups=(32, 64, 128)):
    if weight.ndim != 2 or weight.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError('weight must be floating-point [N,K]')
    n, k = weight.shape
    if (groups and group_size not in groups) or n == 0 or k == 0 or k % group_size or group_size % 2:
        raise ValueError('positive dimensions; group 32/64/128 must divide K')


@torch.no_grad()
def quantize_int4(weight, group_size=128, chunk_rows=256):
    """Symmetric RTN int4 (reference ``quantization.py:35-62``): per group,
    ``scale = absmax/7`` (1 for a zero group), ``q = clamp(round(w/scale), -7, 7)``,
    stored as two's-complement nibbles, low nibble = even k."""
    _check_weight(weight, group_size)
    if chunk_rows <= 0:
        raise ValueError('chunk_rows must be positive')
    n, k = weight.shape
    data = torch.empty((n, k // 2), device=weight.device, dtype=torch.uint8)
    scales = torch.empty((n, k // group_size), device=weight.device, dtype=torch.float32)
    for lo in range(0, n, chunk_rows):
        block = weight[lo:lo + chunk_rows].contiguous()
        if not torch.isfinite(block).all().item():
            raise ValueError('weights must be finite')
        rows = block.shape[0]
        if block.is_cuda:
            with torch.cuda.device(block.device):
                N.check(N.lib().kl_quantize_w4(
                    N.ptr(block), N.act_dtype_code(block.dtype), rows, k, group_size, N.KL_W4_SYM,
                    N.ptr(data[lo:lo + rows]), N.ptr(scales[lo:lo + rows]), None,
                    N.stream_handle(block.device)), ValueError)
            continue
        grouped = block.float().reshape(rows, k // group_size, group_size)
        scale = grouped.abs().amax(-1) / 7
        scale = torch.where(scale == 0, torch.ones_like(scale), scale)
        q = (grouped / scale[..., None]).round().clamp(-7, 7).to(torch.int16).reshape(rows, k)
        nib = q & 15
        data[lo:lo + rows] = (nib[:, 0::2] | (nib[:, 1::2] << 4)).to(torch.uint8)
        scales[lo:lo + rows] = scale
    return PackedInt4(data, scales, group_size)


def _unpack(data):
    low, high = data & 15, data >> 4
    return torch.stack((low, high), -1).reshape(data.shape[0], data.shape[1] * 2).to(torch.int16)


def dequantize_int4(packed):
    """Full f32 weights (reference ``quantization.py:65-71``); the fp32 oracle helper."""
    packed.validate()
    codes = _unpack(packed.data)
    signed = torch.where(codes >= 8, codes - 16, codes).float()
    return signed * packed.scales.repeat_interleave(packed.group_size, dim=1)


@torch.no_grad()
def quantize_int4_asym(weight, group_size=128):
    """Asymmetric RTN int4 with bf16 scale and zero point.

    Per group: ``scale = bf16((max - min) / 15)`` (1 for a constant group),
    ``zero = clamp(round(-min / scale), 0, 15)``, ``q = clamp(round(w / scale)
    + zero, 0, 15)``; nibbles packed two per byte along K, low nibble = even k.
    """
    _check_weight(weight, group_size, groups=())
    n, k = weight.shape
    w = weight.contiguous()
    data = torch.empty((n, k // 2), device=w.device, dtype=torch.uint8)
    scales = torch.empty((n, k // group_size), device=w.device, dtype=torch.bfloat16)
    zeros = torch.empty_like(scales)
    if w.is_cuda:
        with torch.cuda.device(w.device):
            N.check(N.lib().kl_quantize_w4(N.ptr(w), N.act_dtype_code(w.dtype), n, k, group_size, N.KL_W4_ASYM,
                                           N.ptr(data), N.ptr(scales), N.ptr(zeros), N.stream_handle(w.device)),
                    ValueError)
        return PackedInt4Asym(data, scales, zeros, group_size)
    g = w.float().reshape(n, k // group_size, group_size)
    lo, hi = g.amin(-1), g.amax(-1)
    scale = (hi - lo) / 15
    scale = torch.where(scale == 0, torch.ones_like(scale), scale).to(torch.bfloat16)
    sf = scale.float()
    z = (-lo / sf).round().clamp(0, 15)
    q = ((g / sf[..., None]).round() + z[..., None]).clamp(0, 15).to(torch.uint8).reshape(n, k)
    data.copy_(q[:, 0::2] | (q[:, 1::2] << 4))
    scales.copy_(scale)
    zeros.copy_(z.to(torch.bfloat16))
    return PackedInt4Asym(data, scales, zeros, group_size)


def dequantize_int4_asym(packed: PackedInt4Asym):
    packed.validate()
    q = _unpack(packed.data).float()
    s = packed.scales.float().repeat_interleave(packed.group_size, dim=1)
    z = packed.zeros.float().repeat_interleave(packed.group_size, dim=1)
    return (q - z) * s
