"""Install the quantized linear into a Qwen-style decoder (``transformers``
``Qwen3ForCausalLM`` module layout).

Restates the module patches of the reference's
``profiling/decode_stage2_ablation.py:78-143`` for this package's kernels:

* Q, K and V run as ONE fused launch over the row-concatenated weight.  The
  ``q_proj`` call computes all three and the ``k_proj`` / ``v_proj`` calls that
  follow it in the attention forward return their slices; any other call order
  raises ``RuntimeError`` (the reference's rule, :103-110).
* gate and up run as ONE launch with the SwiGLU epilogue fused
  (``mlp.forward`` becomes ``down(silu(gate) * up)``).
* o_proj, down_proj and (optionally) lm_head become :class:`QuantLinear`.
* Every replaced module keeps a ``weight`` attribute: a :class:`QuantWeight`
  (no dense values) over its rows of the packed matrix.  ``torch.cat`` of the
  Q/K/V (or gate/up) weights gives back the fused packed matrix without a copy
  and ``F.linear`` on it runs the quantized kernel, so the reference's serving
  executor (``serving/qwen_executor.py:90-108`` builds its fused weights that
  way; ``:171-174,227-237`` call them) runs on the quantized kernels unchanged;
  :func:`install_quantized_executor` covers an executor built before the
  install.

Unlike the reference adapter, every batch size runs on the quantized kernels
(decode M <= 64 on the HBM-bound path, prefill on the tensor-core path), and
the dense projection weights are released, not retained.  Layers and formats
come from a :class:`~.kernel_policy.QwenKernelPolicy` or from arguments.
"""
from __future__ import annotations

import types

import torch
from torch import nn

from .linear import QuantLinear, quant_linear
from .quant_tensor import QuantWeight

FORMATS = ("w8_row", "w4_asym", "w4_sym")


class _FusedQKV:
    """Shared state of one attention block's fused QKV projection."""

    def __init__(self, weight: QuantLinear, sizes):
        self.weight = weight
        self.sizes = tuple(int(s) for s in sizes)
        self.offsets = [sum(self.sizes[:i]) for i in range(len(self.sizes) + 1)]
        self.pending: dict[int, torch.Tensor] = {}

    def reset(self, module, args):
        self.pending.clear()


class QKVSlice(nn.Module):
    """Stands in for q_proj (slot 0), k_proj (1) or v_proj (2)."""

    def __init__(self, fused: _FusedQKV, slot: int, in_features: int):
        super().__init__()
        self.fused = fused
        self.slot = slot
        self.in_features = in_features
        self.out_features = fused.sizes[slot]

    @property
    def weight(self) -> QuantWeight:
        """This projection's rows of the fused packed matrix (no dense values)."""
        f = self.fused
        return f.weight.weight.slice_rows(f.offsets[self.slot], f.offsets[self.slot + 1])

    def forward(self, x):
        f = self.fused
        if self.slot == 0:
            outputs = f.weight(x).split(f.sizes, dim=-1)
            f.pending.clear()
            f.pending.update(enumerate(outputs))
        if self.slot not in f.pending:
            raise RuntimeError("unexpected Qwen Q/K/V call order")
        return f.pending.pop(self.slot)

    def extra_repr(self):
        return f"slot={self.slot}, out_features={self.out_features}, fused={self.fused.weight.format}"


class RowSlice(nn.Module):
    """gate_proj or up_proj after the install: rows ``[lo, hi)`` of the fused
    gate_up matrix.  The MLP's forward runs the fused launch; this module keeps
    the attribute (and a direct call computes just its rows)."""

    def __init__(self, fused: QuantLinear, lo: int, hi: int):
        super().__init__()
        self.fused = fused
        self.lo, self.hi = lo, hi
        self.in_features = fused.in_features
        self.out_features = hi - lo

    @property
    def weight(self) -> QuantWeight:
        return self.fused.weight.slice_rows(self.lo, self.hi)

    def forward(self, x):
        return quant_linear(x, self.weight.packed)

    def extra_repr(self):
        return f"rows=[{self.lo}, {self.hi}), fused={self.fused.format}"


def _check_bias_free(*modules):
    if any(getattr(m, "bias", None) is not None for m in modules):
        raise ValueError("Qwen bias-free projections required")


def _mlp_forward(self, x):
    return self.down_proj(quant_linear(x, self.kl_gate_up.weight_q, swiglu=True))


def install_quantized_projections(model, policy=None, *, fmt: str = "w8_row", layers=None, lm_head=None,
                                  group_size: int = 128) -> dict:
    """Replace the projections of the selected decoder layers (and optionally the
    lm_head) with quantized ones.  Returns (and stores as ``model._kl_b200_info``)
    a summary: modules replaced, packed bytes, dense bytes released.

    ``policy`` (a QwenKernelPolicy) selects layers and formats through its
    ``w8a16_layers`` / ``w4a16_layers`` / ``quantized_lm_head``; otherwise
    ``layers`` (default: all) are quantized as ``fmt`` and ``lm_head`` names the
    head's format (None keeps it dense).
    """
    decoder = model.model.layers
    count = len(decoder)
    if policy is not None:
        plan = {i: policy.layer_format(i) for i in range(count)}
        head_fmt = policy.quantized_lm_head
    else:
        if fmt not in FORMATS:
            raise ValueError(f"unknown format {fmt!r}")
        chosen = range(count) if layers is None else [int(i) for i in layers]
        if any(i < 0 or i >= count for i in chosen):
            raise ValueError("quantized layer index out of range")
        plan = {i: (fmt if i in set(chosen) else None) for i in range(count)}
        head_fmt = lm_head
    if head_fmt is not None and head_fmt not in FORMATS:
        raise ValueError(f"unknown lm_head format {head_fmt!r}")

    def quantize(key, dense, f):
        return QuantLinear.from_weight(dense(), f, group_size)

    return _install(model, plan, head_fmt, quantize)


def _install(model, plan: dict, head_fmt, make) -> dict:
    """Replace the projections named by ``plan`` (layer -> format or None) and
    the lm_head (``head_fmt``).  ``make(key, dense, fmt)`` returns the
    :class:`QuantLinear` for one projection; ``key`` is its name in a packed
    store (``layers.<i>.qkv|o|gate_up|down`` or ``lm_head``) and ``dense()``
    returns the dense weight it replaces (rows of Q, K, V or gate, up
    concatenated)."""
    decoder = model.model.layers
    replaced, packed_bytes, dense_bytes = 0, 0, 0

    def pack(key, dense, f, out_features, in_features):
        nonlocal packed_bytes
        q = make(key, dense, f)
        if (q.out_features, q.in_features) != (out_features, in_features):
            raise ValueError(f"{key}: packed weight is {q.out_features}x{q.in_features}, "
                             f"the module needs {out_features}x{in_features}")
        packed_bytes += q.weight_q.storage_bytes
        return q

    def released(*modules):
        nonlocal dense_bytes
        for m in modules:
            w = m.weight
            if w.device.type != "meta":
                dense_bytes += w.numel() * w.element_size()

    with torch.no_grad():
        for index, layer in enumerate(decoder):
            f = plan[index]
            if f is None:
                continue
            attn, mlp = layer.self_attn, layer.mlp
            _check_bias_free(attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, mlp.gate_proj, mlp.up_proj,
                             mlp.down_proj)
            act = getattr(mlp, "act_fn", None)
            if not isinstance(act, nn.SiLU) and getattr(act, "__class__", type(None)).__name__ not in ("SiLU", "SiLUActivation"):
                raise ValueError("the fused gate_up epilogue implements SiLU only")
            q, k, v = attn.q_proj, attn.k_proj, attn.v_proj
            sizes = [m.out_features for m in (q, k, v)]
            in_features = q.in_features
            qkv = pack(f"layers.{index}.qkv", lambda: torch.cat([q.weight, k.weight, v.weight]), f,
                       sum(sizes), in_features)
            gate, up, down, o = mlp.gate_proj, mlp.up_proj, mlp.down_proj, attn.o_proj
            o_q = pack(f"layers.{index}.o", lambda: o.weight, f, o.out_features, o.in_features)
            gate_up = pack(f"layers.{index}.gate_up", lambda: torch.cat([gate.weight, up.weight]), f,
                           gate.out_features + up.out_features, gate.in_features)
            down_q = pack(f"layers.{index}.down", lambda: down.weight, f, down.out_features, down.in_features)
            released(q, k, v, o, gate, up, down)
            fused = _FusedQKV(qkv, sizes)
            attn.kl_qkv = fused.weight
            attn.register_forward_pre_hook(fused.reset)
            attn.q_proj = QKVSlice(fused, 0, in_features)
            attn.k_proj = QKVSlice(fused, 1, in_features)
            attn.v_proj = QKVSlice(fused, 2, in_features)
            attn.o_proj = o_q
            mlp.kl_gate_up = gate_up
            half = gate.out_features
            mlp.gate_proj = RowSlice(gate_up, 0, half)
            mlp.up_proj = RowSlice(gate_up, half, 2 * half)
            mlp.down_proj = down_q
            mlp.forward = types.MethodType(_mlp_forward, mlp)
            replaced += 7
        if head_fmt is not None:
            lm = model.lm_head
            _check_bias_free(lm)
            head = lm.weight
            embed = getattr(getattr(model.model, "embed_tokens", None), "weight", None)
            tied = embed is not None and head.device.type != "meta" and head.data_ptr() == embed.data_ptr()
            model.lm_head = pack("lm_head", lambda: head, head_fmt, lm.out_features, lm.in_features)
            if not tied:                              # a tied embedding still holds the dense matrix
                released(lm)
            replaced += 1

    info = {"linear_modules": replaced, "packed_bytes": packed_bytes, "dense_bytes_released": dense_bytes,
            "layers": {i: f for i, f in plan.items() if f is not None}, "lm_head": head_fmt,
            "layout": "fused QKV (one launch), fused gate_up + SwiGLU (one launch), o, down"
                      + (", lm_head" if head_fmt else "")}
    model._kl_b200_info = info
    return info


def install_quantized_executor(executor, policy=None, **kwargs) -> dict:
    """Quantize the projections of a serving executor's model (the reference's
    ``QwenPagedExecutor``: anything with ``.model`` and, optionally,
    ``enable_fused_projections`` / ``fused_qkv_layers`` / ``fused_mlp_layers``)
    and rebuild fused weights it already prepacked, so that its fused QKV and
    gate_up ``F.linear`` sites run the quantized kernel too.  ``policy`` and
    ``kwargs`` are those of :func:`install_quantized_projections`."""
    info = install_quantized_projections(executor.model, policy, **kwargs)
    if getattr(executor, "_projection_weights", None) is not None:
        executor.enable_fused_projections(qkv=executor.fused_qkv_layers, mlp=executor.fused_mlp_layers)
        info["executor_fused_weights"] = "rebuilt from the quantized modules"
    return info
