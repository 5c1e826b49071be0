"""The quantized linear layer: ``quant_linear`` and the ``QuantLinear`` module.

``quant_linear(x, weight)`` is ``F.linear(x, dequant(weight))`` for any leading
shape of ``x`` -- the call the reference's serving executor and model
adapters make at the QKV / o / gate_up / down / lm_head sites
(``serving/qwen_executor.py:173,227,231-232,238``;
``profiling/decode_stage2_ablation.py:78-143``) -- executed by the native
B200 kernels through ``kl_linear``:

* M <= 64 tokens (decode): the tcgen05 swap-AB GEMM streams the quantised
  weights once (HBM-bound), or the CUDA-core GEMV for formats/shapes the
  tensor-core kernel does not take;
* M > 64 (prefill): the same tcgen05 kernel with 128-token tiles (tensor-bound).

``swiglu=True`` treats the weight as ``[gate; up]`` (gate rows first) and
returns the model-ordered ``silu(gate) * up`` in one launch.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _native as N
from . import ops as _ops  # noqa: F401  (registers torch.ops.kl_b200)
from .activation_int8 import CalibratedInt8, RowwiseInt8, quantize_int8_rowwise
from .quantization import PackedInt4, PackedInt4Asym, quantize_int4, quantize_int4_asym


def weight_spec(weight):
    """(format code, data, scales, zeros, inverse, n, k, group) of a weight object."""
    if isinstance(weight, RowwiseInt8):
        n, k = weight.data.shape
        return N.KL_W8_ROW, weight.data, weight.scales, None, None, n, k, k
    if isinstance(weight, PackedInt4Asym):
        n, k = weight.shape
        return N.KL_W4_ASYM, weight.data, weight.scales, weight.zeros, None, n, k, weight.group_size
    if isinstance(weight, PackedInt4):
        n, k = weight.shape
        return N.KL_W4_SYM, weight.data, weight.scales, None, None, n, k, weight.group_size
    if isinstance(weight, CalibratedInt8) or all(hasattr(weight, a) for a in ("data", "scales", "inverse", "group_size")):
        n, k = weight.data.shape
        return N.KL_W8_GROUP, weight.data, weight.scales, None, weight.inverse, n, k, weight.group_size
    if isinstance(weight, torch.Tensor):
        if weight.dtype != torch.bfloat16:
            raise RuntimeError("BF16 or INT8 weights required")
        n, k = weight.shape
        return N.KL_BF16_DENSE, weight, None, None, None, n, k, k
    raise TypeError(f"unsupported weight type {type(weight).__name__}")


def quant_linear(x: torch.Tensor, weight, *, swiglu: bool = False, out: torch.Tensor | None = None,
                 transposed: bool = False, pdl: bool = False, path: str | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x @ dequant(weight)^T`` (f32 accumulation, output in x's dtype).

    x: [..., K] bf16/f16 CUDA tensor.  Returns [..., N_out] (N_out = N, or N/2
    with ``swiglu``), or [N_out, M] when ``transposed`` (x flattened to [M, K]).
    ``path``: None (automatic), "tc" (tcgen05 only), "simt" (CUDA cores only) or
    "persistent" (the persistent stream-K tcgen05 kernel even for a decode-size
    int8 linear that the single-tile cluster kernel would take).
    ``pdl``: launch with programmatic dependent launch (use inside a chain of
    launches / a CUDA graph to overlap weight prefetch with the previous kernel).
    The launch goes through the registered operator ``torch.ops.kl_b200.linear``
    (``linear_out`` when ``out`` is given).  ``workspace``: a caller-owned
    scratch buffer; by default each (device, stream) pair has its own.
    """
    fmt, data, scales, zeros, inverse, n, k, group = weight_spec(weight)
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError("inference only")
    if not x.is_cuda or data.device != x.device:
        raise RuntimeError("x and the weight must be on the same CUDA device")
    if x.shape[-1] != k:
        raise RuntimeError(f"input K {x.shape[-1]} does not match weight K {k}")
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("activations must be BF16 or FP16")
    lead = x.shape[:-1]
    m = 1
    for d in lead:
        m *= d
    x2 = x.reshape(m, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    n_out = n // 2 if swiglu else n
    shape = (n_out, m) if transposed else (*lead, n_out)
    flags = N.KL_FLAG_PDL if pdl else 0
    if path == "tc":
        flags |= N.KL_FLAG_FORCE_TC
    elif path == "simt":
        flags |= N.KL_FLAG_FORCE_SIMT
    elif path == "persistent":
        flags |= N.KL_FLAG_FORCE_TC | N.KL_FLAG_PERSISTENT
    elif path is not None:
        raise ValueError(f"unknown path {path!r}")
    if out is None:
        y = torch.ops.kl_b200.linear(x2, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags,
                                     workspace)
        return y.view(shape)
    if tuple(out.shape) != tuple(shape) or out.dtype != x.dtype or not out.is_contiguous():
        raise RuntimeError("out has the wrong shape, dtype or layout")
    torch.ops.kl_b200.linear_out(x2, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags,
                                 out.view(shape if transposed else (m, n_out)), workspace)
    return out


def lm_head_topk(x: torch.Tensor, weight, k: int = 1, *, index_offset: int = 0, packed: bool = False):
    """Top-``k`` rows of ``x @ dequant(weight)^T`` per token without writing the
    logits: the tcgen05 GEMM's epilogue keeps each 128-row tile's best
    candidates and a merge kernel reduces them (the reference's fused head,
    ``learning/09_int4/kernels.py:37-50,77-99``, for M tokens and the int8 row
    format).  Values are the logits rounded to x's dtype, as f32, descending;
    ties go to the lower row.  Returns ``(values f32 [M, k], ids int64 [M, k])``
    with ids offset by ``index_offset`` (a vocabulary shard's first row), or
    with ``packed`` one int64 ``[M, k]`` tensor of ``id << 32 | value bits``.
    x: [..., K] bf16; weight: int8 row format, or 4-bit with groups of 128
    (at most 64 tokens)."""
    fmt, data, scales, zeros, inverse, n, kdim, group = weight_spec(weight)
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError("inference only")
    if not x.is_cuda or data.device != x.device:
        raise RuntimeError("x and the weight must be on the same CUDA device")
    if x.shape[-1] != kdim or x.dtype != torch.bfloat16:
        raise RuntimeError(f"x must be bf16 [..., {kdim}]")
    if not 1 <= k <= min(8, n):
        raise ValueError("k must be between 1 and min(8, vocabulary)")
    x2 = x.reshape(-1, kdim)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    values, ids = torch.ops.kl_b200.linear_topk(x2, data, scales, zeros, fmt, group, k, index_offset, packed)
    return ids if packed else (values, ids)


class QuantLinear(nn.Module):
    """Bias-free ``nn.Linear`` replacement holding quantised weights only.

    Formats: ``"w8_row"`` (int8 + bf16 per-row scale),
    ``"w4_asym"`` (group-128 asymmetric int4),
    ``"w4_sym"`` (the reference's symmetric int4).  ``swiglu=True`` makes the
    module compute ``silu(gate) * up`` from a stacked ``[gate; up]`` weight.
    """

    def __init__(self, weight, *, swiglu: bool = False):
        super().__init__()
        self.weight_q = weight
        self.swiglu = swiglu
        fmt, data, *_rest = weight_spec(weight)
        n, k = _rest[3], _rest[4]
        self.in_features = k
        self.out_features = n // 2 if swiglu else n
        self.format = fmt

    @classmethod
    def from_weight(cls, weight: torch.Tensor, fmt: str = "w8_row", group_size: int = 128, *, swiglu: bool = False):
        w = weight.detach()
        if fmt == "w8_row":
            q = quantize_int8_rowwise(w)
        elif fmt == "w4_asym":
            q = quantize_int4_asym(w, group_size)
        elif fmt == "w4_sym":
            q = quantize_int4(w, group_size)
        else:
            raise ValueError(f"unknown format {fmt!r}")
        return cls(q, swiglu=swiglu)

    @classmethod
    def from_linear(cls, linear: nn.Linear, fmt: str = "w8_row", group_size: int = 128):
        if linear.bias is not None:
            raise ValueError("bias-free projections required")
        return cls.from_weight(linear.weight, fmt, group_size)

    @property
    def weight(self):
        """The packed matrix as a :class:`~.quant_tensor.QuantWeight` (``F.linear``
        and ``torch.cat`` work on it; it has no dense values)."""
        from .quant_tensor import QuantWeight
        qw = self.__dict__.get("_qweight")
        if qw is None or qw.packed is not self.weight_q:
            qw = QuantWeight(self.weight_q)
            self.__dict__["_qweight"] = qw
        return qw

    def forward(self, x):
        return quant_linear(x, self.weight_q, swiglu=self.swiglu)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, format={self.format}, swiglu={self.swiglu}"


class GroupedLinear:
    """Many independent quantized linears run by ONE persistent tcgen05 launch.

    ``GroupedLinear([(x0, w0, y0), (x1, w1, y1), ...])`` fixes the buffers (the
    problem table holds TMA descriptors of these exact tensors) and ``run()``
    computes every ``y_i = x_i @ dequant(w_i)^T`` with a single kernel that
    streams the weights of all problems through one stream-K partition -- no
    launch gaps between problems.  All weights share one format (KL_W8_ROW or
    a group-128 4-bit format); SwiGLU applies to all problems or none.
    Capture ``run()`` in a CUDA graph for repeated use.

    ``mma``: ``"int8"`` feeds int8 row-scale weights to the tensor core
    unconverted (``kind::i8``) after a digits pass that writes each token row
    as a power-of-two scale and three int8 planes (``x = s (65536 h + 256 m +
    l)``: exact for activations within a factor 2^14 of the row's largest,
    else within ``s / 2``); ``"bf16"`` converts the weights to bf16 in the
    kernel.
    Groups whose every problem has at least 256 tokens (int8 row weights,
    K a multiple of 64) run on the CTA-pair prefill kernel instead, the tiles
    of all problems in one launch (unless ``mma="int8"``).
    For asymmetric 4-bit group-128 weights (at most 16 tokens) the int8 mode
    converts each nibble to the int8 ``q - z`` instead of bf16; it measured
    slower than the bf16 mode on the config 3 set (157-164 against 101 us), so
    ``"auto"`` does not take it.
    ``"auto"`` (default) takes ``"int8"`` for bf16 activations with int8 row
    weights and at most 8 tokens per problem, else ``"bf16"``: the three
    digit planes make the int8 MMA 3 tokens wide per token, which costs more
    tensor time than the bf16 conversion saves once tiles are 16 tokens or
    wider (measured on the config 1 set: 101 against 108 us at M = 1, 163
    against 148 us at M = 64).
    """

    def __init__(self, problems, *, swiglu: bool = False, mma: str = "auto"):
        import ctypes
        if not problems:
            raise ValueError("at least one problem required")
        specs = [weight_spec(w) for _, w, _ in problems]
        fmt = specs[0][0]
        if any(s[0] != fmt for s in specs):
            raise ValueError("all problems must share one weight format")
        x0 = problems[0][0]
        self.device = x0.device
        self.problems = problems              # keep the tensors alive
        arr = (N.KlProblem * len(problems))()
        for i, ((x, w, y), spec) in enumerate(zip(problems, specs)):
            _, data, scales, zeros, _inv, n, k, group = spec
            m = x.numel() // k
            n_out = n // 2 if swiglu else n
            if x.dtype != x0.dtype or not x.is_contiguous() or x.device != self.device or x.shape[-1] != k:
                raise ValueError(f"problem {i}: x must be contiguous [.., {k}] {x0.dtype} on {self.device}")
            if y.dtype != x.dtype or not y.is_contiguous() or y.numel() != m * n_out:
                raise ValueError(f"problem {i}: y must be contiguous with {m}x{n_out} elements")
            arr[i] = N.KlProblem(x.data_ptr(), data.data_ptr(), scales.data_ptr(),
                                 zeros.data_ptr() if zeros is not None else None, y.data_ptr(), m, n, k, group)
        lib = N.lib()
        nbytes = lib.kl_grouped_table_bytes(len(problems))
        if nbytes == 0:
            raise ValueError("too many problems for one grouped launch")
        if mma not in ("auto", "int8", "bf16"):
            raise ValueError(f"mma must be 'auto', 'int8' or 'bf16', not {mma!r}")
        if mma == "auto":
            max_m = max(x.numel() // spec[6] for (x, _, _), spec in zip(problems, specs))
            mma = "int8" if (fmt == N.KL_W8_ROW and x0.dtype == torch.bfloat16 and max_m <= 8) else "bf16"
        self.mma = mma
        flags = N.KL_GROUPED_INT8_MMA if mma == "int8" else 0
        self._digits = None
        dptr, dbytes = None, 0
        if flags:
            dbytes = lib.kl_grouped_digits_bytes(arr, len(problems), flags)
            if dbytes == 0:
                raise ValueError("no digits layout for these problems")
            self._digits = torch.empty(dbytes + 256, dtype=torch.uint8, device=self.device)
            dptr = self._digits.data_ptr() + (-self._digits.data_ptr()) % 256
        self._host = (ctypes.c_uint8 * nbytes)()
        N.check(lib.kl_grouped_encode_ex(arr, len(problems), N.act_dtype_code(x0.dtype), fmt, int(swiglu), flags,
                                         dptr, dbytes, self._host, nbytes))
        host_t = torch.frombuffer(self._host, dtype=torch.uint8)
        self._device = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        off = (-self._device.data_ptr()) % 256
        self._dev_view = self._device[off:off + nbytes]
        self._dev_view.copy_(host_t)
        with torch.cuda.device(self.device):
            self._ws_bytes = lib.kl_grouped_workspace_bytes(self._host)
            N.workspace(self.device, self._ws_bytes)
        torch.cuda.current_stream(self.device).synchronize()

    def run(self, *, pdl: bool = False, workspace: torch.Tensor | None = None):
        lib = N.lib()
        ws = workspace if workspace is not None else N.workspace(self.device, self._ws_bytes)
        ws_bytes = 0 if ws is None else ws.numel() * ws.element_size()
        with torch.cuda.device(self.device):
            N.check(lib.kl_linear_grouped(self._host, N.ptr(self._dev_view), N.ptr(ws), ws_bytes,
                                          N.KL_FLAG_PDL if pdl else 0, N.stream_handle(self.device)))
