"""torch custom ops over the C ABI: ``torch.ops.kl_b200.*``.

The reference exposes its decode projection as a compiled torch extension op
(``learning/10_cuda_decode/warp_gemv.cu:91``, JIT-loaded by
``cuda_decode.py:9-14``).  Here the same role is played by operators
registered with ``torch.library``: each has a CUDA kernel that calls
``libkl_b200.so`` through ``_native`` (plain pointers, sizes and the current
stream) and a fake kernel that only computes the output's shape and dtype, so
the ops are visible to ``torch.ops``, FakeTensor shape propagation,
``torch.compile`` and ``torch.export``.

Operators (``x`` 2-D and contiguous; ``data`` is the weight storage:
int8 ``[N, K]``, packed nibbles uint8 ``[N, K/2]`` or bf16 ``[N, K]``):

* ``linear(x, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags) -> y``
* ``linear_out(..., out)`` -- the same into a caller-owned ``out`` (CUDA graphs)
* ``linear_topk(x, data, scales, zeros, fmt, group, top_k, index_offset, packed)
  -> (values, ids)`` -- the fused lm_head top-k (no logits are written)
* ``project(x, w, scales, inverse, group, warps, persistent, swiglu) -> y`` --
  the reference op's signature (``warp_gemv.cu:56-58``)
* ``int4_gemv(x, data, scales, group, block_n) -> y`` and
  ``int4_lm_head_topk(x, data, scales, group, top_k, block_n) -> (values, ids)``
  (``learning/09_int4/kernels.py:67-99``)

The dispatcher adds about 3 us of host time per call over a plain Python call;
a CUDA graph removes it.  Validation with the reference's exception types
stays in the Python functions that call these ops (``quant_linear``,
``project``, ``int4_gemv``, ``int4_lm_head_topk``); the CUDA kernels raise
``NativeError`` (a ``RuntimeError``) on a non-OK status from the library.
"""
from __future__ import annotations

import torch
from torch.library import Library

from . import _native as N

_lib = Library("kl_b200", "DEF")
_lib.define("linear(Tensor x, Tensor data, Tensor? scales, Tensor? zeros, Tensor? inverse, int fmt, int group, "
            "bool swiglu=False, bool transposed=False, int flags=0, Tensor? workspace=None) -> Tensor")
_lib.define("linear_out(Tensor x, Tensor data, Tensor? scales, Tensor? zeros, Tensor? inverse, int fmt, int group, "
            "bool swiglu, bool transposed, int flags, Tensor(a!) out, Tensor? workspace=None) -> ()")
_lib.define("project(Tensor x, Tensor w, Tensor? scales, Tensor? inverse, int group, int warps, bool persistent, "
            "bool swiglu) -> Tensor")
_lib.define("linear_topk(Tensor x, Tensor data, Tensor? scales, Tensor? zeros, int fmt, int group, int top_k, "
            "int index_offset=0, bool packed=False) -> (Tensor, Tensor)")
_lib.define("int4_gemv(Tensor x, Tensor data, Tensor scales, int group, int block_n) -> Tensor")
_lib.define("int4_lm_head_topk(Tensor x, Tensor data, Tensor scales, int group, int top_k, int block_n) "
            "-> (Tensor, Tensor)")


def _linear_shape(x, data, fmt, swiglu, transposed):
    n = data.shape[0]
    n_out = n // 2 if swiglu else n
    return (n_out, x.shape[0]) if transposed else (x.shape[0], n_out)


# ---- linear -------------------------------------------------------------------
def _linear_out_cuda(x, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags, out,
                     workspace=None):
    m, k = x.shape
    n = data.shape[0]
    if m == 0:
        return
    if transposed:
        flags |= N.KL_FLAG_Y_TRANSPOSED
    lib = N.lib()
    with torch.cuda.device(x.device):
        if workspace is None:
            need = lib.kl_linear_workspace_bytes(m, n, k, fmt, int(swiglu), flags)
            ws = N.workspace(x.device, need, stream=torch.cuda.current_stream(x.device))
        else:
            ws = workspace
        N.check(lib.kl_linear(
            N.ptr(x), N.act_dtype_code(x.dtype), m, k, N.ptr(data), fmt, n, group,
            N.ptr(scales), N.ptr(zeros), N.ptr(inverse), int(swiglu), N.ptr(out),
            N.ptr(ws), 0 if ws is None else ws.numel() * ws.element_size(), flags,
            N.stream_handle(x.device)))


def _linear_cuda(x, data, scales, zeros, inverse, fmt, group, swiglu=False, transposed=False, flags=0,
                 workspace=None):
    out = torch.empty(_linear_shape(x, data, fmt, swiglu, transposed), dtype=x.dtype, device=x.device)
    _linear_out_cuda(x, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags, out, workspace)
    return out


_lib.impl("linear", _linear_cuda, "CUDA")
_lib.impl("linear_out", _linear_out_cuda, "CUDA")


@torch.library.register_fake("kl_b200::linear")
def _linear_fake(x, data, scales, zeros, inverse, fmt, group, swiglu=False, transposed=False, flags=0,
                 workspace=None):
    return x.new_empty(_linear_shape(x, data, fmt, swiglu, transposed))


@torch.library.register_fake("kl_b200::linear_out")
def _linear_out_fake(x, data, scales, zeros, inverse, fmt, group, swiglu, transposed, flags, out, workspace=None):
    return None


# ---- fused lm_head top-k ------------------------------------------------------------
def _linear_topk_cuda(x, data, scales, zeros, fmt, group, top_k, index_offset=0, packed=False):
    m, k = x.shape
    n = data.shape[0]
    lib = N.lib()
    ids = torch.empty(m, top_k, dtype=torch.int64, device=x.device)
    values = torch.empty(0 if packed else m * top_k, dtype=torch.float32, device=x.device).view(-1, top_k)
    with torch.cuda.device(x.device):
        need = lib.kl_linear_topk_workspace_bytes(m, n, k, fmt, top_k)
        ws = N.workspace(x.device, need, stream=torch.cuda.current_stream(x.device))
        N.check(lib.kl_linear_topk(N.ptr(x), N.act_dtype_code(x.dtype), m, k, N.ptr(data), fmt, n, group,
                                   N.ptr(scales), N.ptr(zeros), top_k, index_offset,
                                   None if packed else N.ptr(values), N.ptr(ids), N.ptr(ws),
                                   0 if ws is None else ws.numel(), 0, N.stream_handle(x.device)))
    return values, ids


_lib.impl("linear_topk", _linear_topk_cuda, "CUDA")


@torch.library.register_fake("kl_b200::linear_topk")
def _linear_topk_fake(x, data, scales, zeros, fmt, group, top_k, index_offset=0, packed=False):
    m = x.shape[0]
    return x.new_empty((0 if packed else m, top_k), dtype=torch.float32), x.new_empty((m, top_k), dtype=torch.int64)


# ---- project (the reference op) ---------------------------------------------------
def _project_cuda(x, w, scales, inverse, group, warps, persistent, swiglu):
    n, k = w.shape
    y = torch.empty(n // 2 if swiglu else n, dtype=torch.bfloat16, device=x.device)
    int8 = w.dtype == torch.int8
    with torch.cuda.device(x.device):
        N.check(N.lib().kl_project(N.ptr(x), k, N.ptr(w), int(int8), N.ptr(scales) if int8 else None,
                                   N.ptr(inverse) if int8 else None, n, group if int8 else 128, warps,
                                   int(persistent), int(swiglu), N.ptr(y), None, 0, N.stream_handle(x.device)))
    return y


_lib.impl("project", _project_cuda, "CUDA")


@torch.library.register_fake("kl_b200::project")
def _project_fake(x, w, scales, inverse, group, warps, persistent, swiglu):
    return x.new_empty(w.shape[0] // 2 if swiglu else w.shape[0], dtype=torch.bfloat16)


# ---- int4 -------------------------------------------------------------------------
def _int4_gemv_cuda(x, data, scales, group, block_n):
    n, k = data.shape[0], x.numel()
    if group == 128 and k % 128 == 0 and x.dtype == torch.bfloat16:
        # the tcgen05 kernel, on the plan the fused head uses: its values are
        # exactly the logits this returns (the reference shares _project too)
        return _linear_cuda(x.view(1, k), data, scales, None, None, N.KL_W4_SYM, group).view(n)
    y = torch.empty(n, device=x.device, dtype=x.dtype)
    with torch.cuda.device(x.device):
        N.check(N.lib().kl_int4_gemv(N.ptr(x), N.act_dtype_code(x.dtype), k, N.ptr(data), N.ptr(scales), n,
                                     group, block_n, N.ptr(y), N.stream_handle(x.device)), ValueError)
    return y


def _int4_head_cuda(x, data, scales, group, top_k, block_n):
    n, k = data.shape[0], x.numel()
    lib = N.lib()
    values = torch.empty(top_k, device=x.device, dtype=torch.float32)
    ids = torch.empty(top_k, device=x.device, dtype=torch.int64)
    with torch.cuda.device(x.device):
        need = max(lib.kl_int4_lm_head_topk_workspace_bytes(n, top_k, block_n),
                   lib.kl_linear_topk_workspace_bytes(1, n, k, N.KL_W4_SYM, top_k))
        ws = N.workspace(x.device, need, stream=torch.cuda.current_stream(x.device))
        N.check(lib.kl_int4_lm_head_topk(N.ptr(x), N.act_dtype_code(x.dtype), k, N.ptr(data), N.ptr(scales), n,
                                         group, top_k, block_n, N.ptr(values), N.ptr(ids), N.ptr(ws), ws.numel(),
                                         N.stream_handle(x.device)), ValueError)
    return values, ids


_lib.impl("int4_gemv", _int4_gemv_cuda, "CUDA")
_lib.impl("int4_lm_head_topk", _int4_head_cuda, "CUDA")


@torch.library.register_fake("kl_b200::int4_gemv")
def _int4_gemv_fake(x, data, scales, group, block_n):
    return x.new_empty(data.shape[0])


@torch.library.register_fake("kl_b200::int4_lm_head_topk")
def _int4_head_fake(x, data, scales, group, top_k, block_n):
    return x.new_empty(top_k, dtype=torch.float32), x.new_empty(top_k, dtype=torch.int64)


OPS = ("linear", "linear_out", "linear_topk", "project", "int4_gemv", "int4_lm_head_topk")
