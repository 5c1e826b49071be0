"""Capability-based kernel selection for Qwen models, with the quantized linear.

Mirrors the dispatch contract of the reference's ``serving/kernel_policy.py``
(``DeviceCapabilities``, ``ModelSignature``, ``QwenKernelPolicy``,
``select_qwen_policy``, ``load_qwen_policy``; lines 11-98 there):

* a model whose signature differs from the profile's, or a GPU architecture
  without a row whose ``quality_gate_passed`` is true, gets the exact
  ``fallback`` policy (no fused or direct kernels, ``calibrated`` false);
* a row naming an out-of-range layer, a non-power-of-two block size or an
  attention tile outside {64, 128, 256} raises ``ValueError``.

Quantized projections are enabled by new optional row keys, so profiles
written for the reference stay valid and select exactly what they selected:

* ``w8a16_layers`` / ``w4a16_layers``: decoder layers whose QKV, o, gate_up and
  down projections run on the int8 row-scale / 4-bit group-128 kernels (the two
  sets must not overlap);
* ``quantized_lm_head``: ``"w8_row"``, ``"w4_asym"`` or absent.

The attention-related fields are carried through unchanged for the caller;
this package does not implement attention.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch

DEFAULT_PROFILES = Path(__file__).with_name("calibrations") / "qwen3_0.6b.json"
LM_HEAD_FORMATS = ("w8_row", "w4_asym")


@dataclass(frozen=True)
class DeviceCapabilities:
    name: str
    major: int
    minor: int
    multiprocessors: int
    warp_size: int
    total_memory: int

    @property
    def architecture(self):
        return f"sm{self.major}{self.minor}"


@dataclass(frozen=True)
class ModelSignature:
    layers: int
    hidden_size: int
    attention_heads: int
    kv_heads: int
    head_dim: int


@dataclass(frozen=True)
class QwenKernelPolicy:
    profile: str
    architecture: str
    block_size: int
    attention_tile: int
    direct_attention_layers: frozenset
    fused_gather: bool
    native_gqa: bool
    fused_qkv_layers: frozenset
    fused_mlp_layers: frozenset
    calibrated: bool
    reason: str
    # quantized linear (absent from reference profiles: nothing quantized)
    w8a16_layers: frozenset = frozenset()
    w4a16_layers: frozenset = frozenset()
    quantized_lm_head: str | None = None

    def layer_format(self, index: int) -> str | None:
        """Weight format of decoder layer ``index``'s projections, or None (dense)."""
        if index in self.w8a16_layers:
            return "w8_row"
        if index in self.w4a16_layers:
            return "w4_asym"
        return None


def _fallback(capabilities: DeviceCapabilities, reason: str) -> QwenKernelPolicy:
    return QwenKernelPolicy("fallback", capabilities.architecture, 16, 128, frozenset(), False, False,
                            frozenset(), frozenset(), False, reason)


def detect_cuda_capabilities(device=None) -> DeviceCapabilities:
    device = torch.device("cuda" if device is None else device)
    if device.type != "cuda" or not torch.cuda.is_available():
        raise ValueError("CUDA device required")
    props = torch.cuda.get_device_properties(device)
    major, minor = torch.cuda.get_device_capability(device)
    return DeviceCapabilities(props.name, major, minor, props.multi_processor_count, props.warp_size,
                              props.total_memory)


def qwen_signature(model) -> ModelSignature:
    config = model.config
    return ModelSignature(len(model.model.layers), config.hidden_size, config.num_attention_heads,
                          config.num_key_value_heads, config.head_dim)


def _layer_set(row: dict, key: str) -> frozenset:
    return frozenset(int(x) for x in row.get(key, ()))


def select_qwen_policy(capabilities: DeviceCapabilities, signature: ModelSignature, profiles: dict) -> QwenKernelPolicy:
    expected = profiles["model_signature"]
    actual = {"layers": signature.layers, "hidden_size": signature.hidden_size,
              "attention_heads": signature.attention_heads, "kv_heads": signature.kv_heads,
              "head_dim": signature.head_dim}
    if actual != expected:
        return _fallback(capabilities, "model signature is not calibrated")
    row = profiles.get("architectures", {}).get(capabilities.architecture)
    if row is None or not row.get("quality_gate_passed", False):
        return _fallback(capabilities, "GPU architecture has no accepted quality profile")
    direct = _layer_set(row, "direct_attention_layers")
    qkv = _layer_set(row, "fused_qkv_layers")
    mlp = _layer_set(row, "fused_mlp_layers")
    w8 = _layer_set(row, "w8a16_layers")
    w4 = _layer_set(row, "w4a16_layers")
    if any(x < 0 or x >= signature.layers for x in direct | qkv | mlp | w8 | w4):
        raise ValueError("calibration contains an invalid layer index")
    if w8 & w4:
        raise ValueError("calibration assigns a layer to both w8a16_layers and w4a16_layers")
    block = int(row.get("block_size", 16))
    tile = int(row.get("attention_tile", 128))
    if block <= 0 or block & (block - 1) or tile not in (64, 128, 256):
        raise ValueError("calibration contains an invalid block/tile size")
    head = row.get("quantized_lm_head")
    if head is not None and head not in LM_HEAD_FORMATS:
        raise ValueError(f"calibration contains an unknown lm_head format {head!r}")
    return QwenKernelPolicy(row.get("name", capabilities.architecture), capabilities.architecture, block, tile,
                            direct, bool(row.get("fused_gather", False)), bool(row.get("native_gqa", False)),
                            qkv, mlp, True, "matched accepted architecture profile", w8, w4, head)


def load_qwen_policy(model, device=None, path=DEFAULT_PROFILES) -> QwenKernelPolicy:
    profiles = json.loads(Path(path).read_text(encoding="utf-8"))
    return select_qwen_policy(detect_cuda_capabilities(device), qwen_signature(model), profiles)
