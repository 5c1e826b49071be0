"""On-disk store of packed (quantized) projection weights.

The reference quantizes at model load and keeps the dense bf16 weights
resident beside the packed ones. Its decode-stage report counts the cost as
455 MB of extra resident memory (``activation_int8.py:10-21`` and
``quantization.py:7-32`` hold the formats). Here a model is quantized once,
its packed tensors are saved, and later loads install them straight into the
module tree. The dense projection weights are then never needed: the model
can be built on the ``meta`` device, because only the modules' shapes are
read.

File layout: one ``torch.save`` dict, read back with ``weights_only=True`` (no
pickled code).

* ``tag``: ``"kl_b200.packed/1"``
* ``layers``: ``{layer index: format}``
* ``lm_head``: format or None
* ``entries``: ``{key: entry}``. Keys are ``layers.<i>.qkv``, ``.o``,
  ``.gate_up``, ``.down`` and ``lm_head``. QKV rows are Q, K, V concatenated;
  gate_up rows are gate then up.
* Each entry holds ``format``, ``data``, ``scales`` and ``zeros`` (4-bit
  asymmetric only), plus ``group_size``.

The tensors are the kernels' own formats, byte for byte:

* ``w8_row``: int8 ``[N, K]`` with bf16 ``[N]`` scales.
* ``w4_asym``: uint8 ``[N, K/2]`` (low nibble = even k) with bf16 scale and
  zero per group.
* ``w4_sym``: the reference's ``PackedInt4``, with f32 group scales.
"""
from __future__ import annotations

import torch

from .activation_int8 import RowwiseInt8
from .adapters import _install
from .linear import QuantLinear
from .quantization import PackedInt4, PackedInt4Asym

TAG = "kl_b200.packed/1"


def _entry(weight) -> dict:
    if isinstance(weight, RowwiseInt8):
        return {"format": "w8_row", "data": weight.data, "scales": weight.scales, "zeros": None, "group_size": 0}
    if isinstance(weight, PackedInt4Asym):
        return {"format": "w4_asym", "data": weight.data, "scales": weight.scales, "zeros": weight.zeros,
                "group_size": int(weight.group_size)}
    if isinstance(weight, PackedInt4):
        return {"format": "w4_sym", "data": weight.data, "scales": weight.scales, "zeros": None,
                "group_size": int(weight.group_size)}
    raise TypeError(f"no packed store format for {type(weight).__name__}")


def _weight(entry: dict, device):
    fmt = entry.get("format")
    data, scales, zeros = (entry[k].to(device) if entry.get(k) is not None else None
                           for k in ("data", "scales", "zeros"))
    if fmt == "w8_row":
        w = RowwiseInt8(data, scales)
    elif fmt == "w4_asym":
        w = PackedInt4Asym(data, scales, zeros, int(entry["group_size"]))
    elif fmt == "w4_sym":
        w = PackedInt4(data, scales, int(entry["group_size"]))
    else:
        raise ValueError(f"unknown packed format {fmt!r}")
    w.validate()
    return w


def export_packed(model) -> dict:
    """The packed weights of a model that ``install_quantized_projections`` (or
    :func:`install_packed`) has rewritten, as a store dict."""
    info = getattr(model, "_kl_b200_info", None)
    if info is None:
        raise ValueError("the model has no quantized projections installed")
    entries = {}
    for index in info["layers"]:
        layer = model.model.layers[index]
        entries[f"layers.{index}.qkv"] = _entry(layer.self_attn.kl_qkv.weight_q)
        entries[f"layers.{index}.o"] = _entry(layer.self_attn.o_proj.weight_q)
        entries[f"layers.{index}.gate_up"] = _entry(layer.mlp.kl_gate_up.weight_q)
        entries[f"layers.{index}.down"] = _entry(layer.mlp.down_proj.weight_q)
    if info["lm_head"] is not None:
        entries["lm_head"] = _entry(model.lm_head.weight_q)
    return {"tag": TAG, "layers": {int(i): f for i, f in info["layers"].items()}, "lm_head": info["lm_head"],
            "entries": entries}


def save_packed(path, store: dict) -> None:
    """Write a store dict (tensors are copied to host memory first)."""
    if store.get("tag") != TAG:
        raise ValueError("not a packed-weight store")
    host = {k: v for k, v in store.items() if k not in ("entries", "device")}
    host["entries"] = {key: {k: (v.detach().cpu().contiguous() if isinstance(v, torch.Tensor) else v)
                             for k, v in e.items()} for key, e in store["entries"].items()}
    torch.save(host, path)


def load_packed(path, device=None) -> dict:
    """Read a store written by :func:`save_packed`.  Its tensors stay in host
    memory; :func:`install_packed` moves them to ``device`` (if given) as it
    builds the modules."""
    store = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(store, dict) or store.get("tag") != TAG:
        raise ValueError(f"{path}: not a {TAG} store")
    store["device"] = device
    return store


def install_packed(model, store: dict, device=None) -> dict:
    """Install the store's packed weights into ``model``: the same module
    rewrite as ``install_quantized_projections`` (fused QKV, fused gate_up +
    SwiGLU, o, down, optionally lm_head), with no quantization and no read of
    the dense projection weights.  Every packed shape is checked against the
    module it replaces (``ValueError`` on a mismatch or a missing entry)."""
    if store.get("tag") != TAG:
        raise ValueError("not a packed-weight store")
    device = device if device is not None else store.get("device")
    entries = store["entries"]
    count = len(model.model.layers)
    layers = {int(i): f for i, f in store["layers"].items()}
    if any(i < 0 or i >= count for i in layers):
        raise ValueError("store names a layer the model does not have")
    plan = {i: layers.get(i) for i in range(count)}

    def load(key, dense, f):
        if key not in entries:
            raise ValueError(f"store has no entry {key!r}")
        e = entries[key]
        if e["format"] != f:
            raise ValueError(f"{key}: stored as {e['format']}, the store's plan says {f}")
        return QuantLinear(_weight(e, device if device is not None else e["data"].device))

    return _install(model, plan, store["lm_head"], load)
