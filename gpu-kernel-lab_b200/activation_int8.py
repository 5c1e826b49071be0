"""W8A16 weight containers and quantisers.

Mirrors the reference's ``learning/10_cuda_decode/activation_int8.py``
(``CalibratedInt8``, ``quantize_int8``, ``dequantize_int8``: same names, fields,
argument meaning and ``ValueError`` behaviour) and adds the per-output-row
format of BASELINE.json config 0 (``RowwiseInt8``).

Quantisation is offline weight packing, not the hot path: the calibrated
search is plain torch on the weight's device, exactly as in the reference
(``activation_int8.py:24-60``); the per-row quantiser runs the native CUDA
kernel for CUDA weights (``kl_quantize_w8_row``) and the same arithmetic in
torch for CPU weights.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as N


@dataclass
class CalibratedInt8:
    """Reference format (``activation_int8.py:10-21``): ``w = q * s[n, k//g] * inverse[k]``."""
    data: torch.Tensor          # int8 [N, K]
    scales: torch.Tensor        # f32 [N, K / group_size]
    inverse: torch.Tensor       # f32 [K]
    group_size: int
    alpha: float
    calibration_mse: float

    @property
    def storage_bytes(self):
        return self.data.numel() + 4 * (self.scales.numel() + self.inverse.numel())

    @property
    def shape(self):
        return tuple(self.data.shape)


@torch.inference_mode()
def quantize_int8(weight, calibration, group_size=128, alphas=(0., .5, 1.)):
    """AWQ-inspired channel-scale search (reference ``activation_int8.py:24-60``).

    For each alpha the channel vector is ``clamp(mean|x|^alpha, 1e-2, 1e2)``
    normalised by ``sqrt(max*min)``; weights times channel are quantised per
    ``group_size`` block of K to ``round(w / (absmax/127))`` in [-127, 127];
    the candidate with the lowest local output MSE on ``calibration`` wins.
    """
    if weight.ndim != 2 or calibration.ndim != 2 or weight.shape[1] != calibration.shape[1]:
        raise ValueError('expected weight[N,K], calibration[T,K]')
    n, k = weight.shape
    if n == 0 or k == 0 or group_size <= 0 or k % group_size or calibration.shape[0] == 0:
        raise ValueError('nonempty tensors and group dividing K required')
    if not alphas or any(a < 0 or a > 1 for a in alphas):
        raise ValueError('nonempty alpha values in [0,1] required')
    if weight.device != calibration.device or not weight.is_floating_point() or not calibration.is_floating_point():
        raise ValueError('colocated floating-point inputs required')
    if not torch.isfinite(weight).all().item() or not torch.isfinite(calibration).all().item():
        raise ValueError('finite inputs required')
    act = calibration.float()
    importance = act.abs().mean(0).clamp_min(1e-4)
    best = None
    for alpha in alphas:
        channel = importance.pow(alpha).clamp(1e-2, 1e2)
        channel /= (channel.max() * channel.min()).sqrt()
        codes = torch.empty((n, k), dtype=torch.int8, device=weight.device)
        scales = torch.empty((n, k // group_size), dtype=torch.float32, device=weight.device)
        sq_err = 0.
        for lo in range(0, n, 256):
            block = weight[lo:lo + 256].float()
            grouped = (block * channel).reshape(block.shape[0], -1, group_size)
            scale = grouped.abs().amax(-1) / 127
            scale = torch.where(scale == 0, torch.ones_like(scale), scale)
            q = (grouped / scale[..., None]).round().clamp(-127, 127).to(torch.int8)
            approx = (q.float() * scale[..., None]).reshape(block.shape) / channel
            sq_err += ((act @ approx.T - act @ block.T).square().sum()).item()
            codes[lo:lo + block.shape[0]] = q.reshape(block.shape)
            scales[lo:lo + block.shape[0]] = scale
        cand = CalibratedInt8(codes, scales, channel.reciprocal().contiguous(), group_size, float(alpha),
                              sq_err / (act.shape[0] * n))
        if best is None or cand.calibration_mse < best.calibration_mse:
            best = cand
    return best


def dequantize_int8(weight):
    """f32 ``q * s * inverse`` (reference ``activation_int8.py:63-64``); any device.

    This is the fp32 oracle helper of the reference API; the GEMM kernels never
    materialise dequantised weights.  ``dequantize_native`` gives the same
    values computed by the CUDA kernel.
    """
    return weight.data.float() * weight.scales.repeat_interleave(weight.group_size, 1) * weight.inverse


@dataclass
class RowwiseInt8:
    """BASELINE.json config 0 format: int8 ``data[N,K]``, bf16 ``scales[N]``, ``w = q * s[n]``."""
    data: torch.Tensor          # int8 [N, K]
    scales: torch.Tensor        # bf16 [N]

    @property
    def shape(self):
        return tuple(self.data.shape)

    @property
    def storage_bytes(self):
        return self.data.numel() + 2 * self.scales.numel()

    def validate(self):
        if self.data.ndim != 2 or self.data.dtype != torch.int8:
            raise ValueError('data must be int8 [N,K]')
        if self.scales.shape != (self.data.shape[0],) or self.scales.dtype != torch.bfloat16:
            raise ValueError('scales must be bf16 [N]')
        if self.data.device != self.scales.device or not self.data.is_contiguous() or not self.scales.is_contiguous():
            raise ValueError('contiguous colocated buffers required')

    def to(self, device):
        return RowwiseInt8(self.data.to(device), self.scales.to(device))


@torch.inference_mode()
def quantize_int8_rowwise(weight):
    """Per-row absmax/127 quantisation with a bf16 scale.

    ``scale = bf16(absmax_n / 127)`` (1 for an all-zero row), then
    ``q = clamp(round_half_even(w / scale), -127, 127)`` with the bf16 scale,
    so that ``q * scale`` is exactly the dequantised weight.
    """
    if weight.ndim != 2 or weight.shape[0] == 0 or weight.shape[1] == 0:
        raise ValueError('weight must be a nonempty [N,K] matrix')
    if not weight.is_floating_point():
        raise ValueError('floating-point weight required')
    w = weight.contiguous()
    n, k = w.shape
    if w.is_cuda:
        if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            w = w.float()
        q = torch.empty((n, k), dtype=torch.int8, device=w.device)
        s = torch.empty(n, dtype=torch.bfloat16, device=w.device)
        with torch.cuda.device(w.device):
            N.check(N.lib().kl_quantize_w8_row(N.ptr(w), N.act_dtype_code(w.dtype), n, k, N.ptr(q), N.ptr(s),
                                               N.stream_handle(w.device)))
        return RowwiseInt8(q, s)
    wf = w.float()
    scale = wf.abs().amax(1) / 127
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    s = scale.to(torch.bfloat16)
    q = (wf / s.float()[:, None]).round().clamp(-127, 127).to(torch.int8)
    return RowwiseInt8(q, s)


def dequantize_int8_rowwise(weight: RowwiseInt8):
    return weight.data.float() * weight.scales.float()[:, None]
