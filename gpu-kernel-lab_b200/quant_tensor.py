"""``QuantWeight``: an ``[N, K]`` weight tensor that exists only in packed form.

Callers that build their own fused weights and call ``F.linear`` on them --
the reference's serving executor does both (``serving/qwen_executor.py:90-108``
concatenates ``q_proj/k_proj/v_proj.weight`` and ``gate_proj/up_proj.weight``
with ``torch.cat``; ``:171-174`` and ``:230-232`` call ``F.linear`` on the
results) -- work unchanged on quantized weights through this tensor subclass:

* ``F.linear(x, w)`` runs ``quant_linear(x, w.packed)`` (``torch.ops.kl_b200``);
* ``torch.cat([w0, w1, ...], dim=0)`` concatenates the packed rows.  Slices of
  one packed matrix that are adjacent and in order (the adapter's Q/K/V and
  gate/up views) give back a view of that matrix: nothing is copied;
* ``.contiguous()``, ``.detach()`` and ``.to(same device)`` return the weight;
  ``shape``, ``dtype``, ``device`` and ``ndim`` read as the dense weight's.

The tensor has no dense storage.  Any other operation raises ``TypeError``
(loudly: nothing falls back to a dense computation).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .activation_int8 import CalibratedInt8, RowwiseInt8
from .quantization import PackedInt4, PackedInt4Asym

_PASS = {torch.Tensor.shape.__get__, torch.Tensor.dtype.__get__, torch.Tensor.device.__get__,
         torch.Tensor.ndim.__get__, torch.Tensor.size, torch.Tensor.dim, torch.Tensor.is_cuda.__get__,
         torch.Tensor.requires_grad.__get__, torch.Tensor.__repr__, torch.Tensor.__format__,
         torch.Tensor.layout.__get__, torch.Tensor.is_sparse.__get__, torch.Tensor.numel}
_SELF = {torch.Tensor.contiguous, torch.Tensor.detach, torch.Tensor.requires_grad_}


def row_slice(packed, lo: int, hi: int):
    """Rows ``[lo, hi)`` of a packed weight, as views of its buffers."""
    if isinstance(packed, RowwiseInt8):
        return RowwiseInt8(packed.data[lo:hi], packed.scales[lo:hi])
    if isinstance(packed, PackedInt4Asym):
        return PackedInt4Asym(packed.data[lo:hi], packed.scales[lo:hi], packed.zeros[lo:hi], packed.group_size)
    if isinstance(packed, PackedInt4):
        return PackedInt4(packed.data[lo:hi], packed.scales[lo:hi], packed.group_size)
    if isinstance(packed, CalibratedInt8):
        return CalibratedInt8(packed.data[lo:hi], packed.scales[lo:hi], packed.inverse, packed.group_size,
                              packed.alpha, packed.calibration_mse)
    raise TypeError(f"unsupported packed weight {type(packed).__name__}")


def concat_rows(parts):
    """Row-concatenation of packed weights of one format (copies the buffers)."""
    first = parts[0]
    if any(type(p) is not type(first) for p in parts):
        raise TypeError("cannot concatenate packed weights of different formats")
    cat = lambda name: torch.cat([getattr(p, name) for p in parts], dim=0)  # noqa: E731
    if isinstance(first, RowwiseInt8):
        return RowwiseInt8(cat("data"), cat("scales"))
    if any(p.group_size != first.group_size for p in parts):
        raise ValueError("cannot concatenate packed weights with different group sizes")
    if isinstance(first, PackedInt4Asym):
        return PackedInt4Asym(cat("data"), cat("scales"), cat("zeros"), first.group_size)
    if isinstance(first, PackedInt4):
        return PackedInt4(cat("data"), cat("scales"), first.group_size)
    if isinstance(first, CalibratedInt8):
        if any(p.inverse is not first.inverse and not torch.equal(p.inverse, first.inverse) for p in parts):
            raise ValueError("calibrated int8 weights with different inverse channel vectors")
        return CalibratedInt8(cat("data"), cat("scales"), first.inverse, first.group_size, first.alpha,
                              first.calibration_mse)
    raise TypeError(f"unsupported packed weight {type(first).__name__}")


class QuantWeight(torch.Tensor):
    """Dense-looking ``[N, K]`` handle on a packed weight (``.packed``).  ``parent``
    and ``rows`` record the packed matrix this one is a row range of, so that
    concatenating adjacent ranges returns a view instead of a copy."""

    @staticmethod
    def __new__(cls, packed, dtype=torch.bfloat16, parent=None, rows=None):
        n, k = packed.shape
        t = torch.Tensor._make_wrapper_subclass(cls, (n, k), dtype=dtype, device=packed.data.device,
                                                requires_grad=False)
        t.packed = packed
        t.parent = parent if parent is not None else packed
        t.rows = rows if rows is not None else (0, n)
        return t

    def __init__(self, packed, dtype=torch.bfloat16, parent=None, rows=None):
        pass

    def slice_rows(self, lo: int, hi: int) -> "QuantWeight":
        base = self.rows[0]
        return QuantWeight(row_slice(self.packed, lo, hi), self.dtype, self.parent, (base + lo, base + hi))

    def __repr__(self, **kwargs):
        return (f"QuantWeight({type(self.packed).__name__}, shape={tuple(self.shape)}, "
                f"device={self.packed.data.device})")

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in _PASS:
            with torch._C.DisableTorchFunctionSubclass():
                return func(*args, **kwargs)
        if func in _SELF:
            return args[0]
        if func is torch.Tensor.to:
            w = args[0]
            target = [a for a in list(args[1:]) + list(kwargs.values()) if isinstance(a, (torch.device, str))]
            if all(torch.device(t) == w.device for t in target) and not any(
                    isinstance(a, torch.dtype) and a != w.dtype for a in list(args[1:]) + list(kwargs.values())):
                return w
            raise TypeError("a quantized weight cannot be moved or cast; re-quantize on the target device")
        if func in (F.linear, torch._C._nn.linear):
            x, w = args[0], args[1]
            bias = args[2] if len(args) > 2 else kwargs.get("bias")
            if not isinstance(w, QuantWeight) or isinstance(x, QuantWeight):
                raise TypeError("F.linear takes the quantized weight as its second argument")
            if bias is not None:
                raise TypeError("quantized projections are bias-free")
            from .linear import quant_linear
            return quant_linear(x, w.packed)
        if func in (torch.cat, torch.concat, torch.concatenate):
            tensors = list(args[0])
            dim = kwargs.get("dim", args[1] if len(args) > 1 else 0)
            if dim not in (0, -2) or not all(isinstance(t, QuantWeight) for t in tensors):
                raise TypeError("quantized weights concatenate along rows (dim 0), with each other only")
            first = tensors[0]
            adjacent = all(t.parent is first.parent for t in tensors) and all(
                a.rows[1] == b.rows[0] for a, b in zip(tensors, tensors[1:]))
            if adjacent:
                lo, hi = first.rows[0], tensors[-1].rows[1]
                return QuantWeight(row_slice(first.parent, lo, hi), first.dtype, first.parent, (lo, hi))
            return QuantWeight(concat_rows([t.packed for t in tensors]), first.dtype)
        raise TypeError(f"{getattr(func, '__name__', func)} is not supported on a quantized weight "
                        "(it has no dense values)")

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        raise TypeError(f"{func} is not supported on a quantized weight (it has no dense values)")
