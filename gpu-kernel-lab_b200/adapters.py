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

FORMATS = ("w8_row", "w4_asym", "w4_sym")


class _FusedQKV:
    """Shared state of one attention block's fused QKV projection."""

    def __init__(self, weight: QuantLinear, sizes):
        self.weight = weight
        self.sizes = tuple(int(s) for s in sizes)
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

    replaced, packed_bytes, dense_bytes = 0, 0, 0

    def pack(weight, f):
        nonlocal packed_bytes, dense_bytes
        q = QuantLinear.from_weight(weight, f, group_size)
        packed_bytes += q.weight_q.storage_bytes
        dense_bytes += weight.numel() * weight.element_size()
        return q

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
            sizes = [m.out_features for m in (attn.q_proj, attn.k_proj, attn.v_proj)]
            in_features = attn.q_proj.in_features
            fused = _FusedQKV(pack(torch.cat([attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight]), f), sizes)
            attn.kl_qkv = fused.weight
            attn.register_forward_pre_hook(fused.reset)
            attn.q_proj = QKVSlice(fused, 0, in_features)
            attn.k_proj = QKVSlice(fused, 1, in_features)
            attn.v_proj = QKVSlice(fused, 2, in_features)
            attn.o_proj = pack(attn.o_proj.weight, f)
            gate_up = pack(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]), f)
            mlp.kl_gate_up = gate_up
            del mlp.gate_proj, mlp.up_proj
            mlp.down_proj = pack(mlp.down_proj.weight, f)
            mlp.forward = types.MethodType(_mlp_forward, mlp)
            replaced += 7
        if head_fmt is not None:
            _check_bias_free(model.lm_head)
            head = model.lm_head.weight
            embed = getattr(getattr(model.model, "embed_tokens", None), "weight", None)
            tied = embed is not None and head.data_ptr() == embed.data_ptr()
            model.lm_head = pack(head, head_fmt)
            if tied:                                  # the embedding still holds the dense matrix
                dense_bytes -= head.numel() * head.element_size()
            replaced += 1

    info = {"linear_modules": replaced, "packed_bytes": packed_bytes, "dense_bytes_released": dense_bytes,
            "layers": {i: f for i, f in plan.items() if f is not None}, "lm_head": head_fmt,
            "layout": "fused QKV (one launch), fused gate_up + SwiGLU (one launch), o, down"
                      + (", lm_head" if head_fmt else "")}
    model._kl_b200_info = info
    return info
