"""The dispatch contract (reference ``serving/kernel_policy.py`` and its tests in
``serving/test_kernel_policy.py``), extended with the quantized-linear keys.
CPU only."""
import json

import pytest

from tests.conftest import load_kl

kl = load_kl()
P = kl.kernel_policy

PROFILES = {
    "model_signature": {"layers": 28, "hidden_size": 1024, "attention_heads": 16, "kv_heads": 8, "head_dim": 128},
    "architectures": {
        "sm89": {"name": "ada", "quality_gate_passed": True, "block_size": 16, "attention_tile": 128,
                 "direct_attention_layers": [24, 25, 26, 27], "fused_gather": True, "native_gqa": True,
                 "fused_qkv_layers": [26, 27], "fused_mlp_layers": list(range(28))},
        "sm100": {"name": "b200", "quality_gate_passed": True, "block_size": 16, "attention_tile": 128,
                  "fused_qkv_layers": list(range(28)), "fused_mlp_layers": list(range(28)),
                  "w8a16_layers": list(range(0, 20)), "w4a16_layers": list(range(20, 28)),
                  "quantized_lm_head": "w8_row"},
        "sm90": {"name": "rejected", "quality_gate_passed": False, "w8a16_layers": [0]},
    },
}
SIGNATURE = P.ModelSignature(28, 1024, 16, 8, 128)


def caps(major, minor):
    return P.DeviceCapabilities("test", major, minor, 148, 32, 180 << 30)


def test_known_architecture_uses_only_calibrated_layers():
    policy = P.select_qwen_policy(caps(8, 9), SIGNATURE, PROFILES)
    assert policy.calibrated and policy.profile == "ada"
    assert policy.direct_attention_layers == frozenset({24, 25, 26, 27})
    assert policy.fused_gather and policy.native_gqa
    assert policy.fused_qkv_layers == frozenset({26, 27})
    assert len(policy.fused_mlp_layers) == 28
    # a reference profile quantizes nothing
    assert not policy.w8a16_layers and not policy.w4a16_layers and policy.quantized_lm_head is None
    assert all(policy.layer_format(i) is None for i in range(28))


def test_unknown_architecture_uses_exact_fallback():
    policy = P.select_qwen_policy(caps(7, 5), SIGNATURE, PROFILES)
    assert not policy.calibrated and not policy.direct_attention_layers
    assert not policy.fused_gather and not policy.native_gqa
    assert not policy.w8a16_layers and policy.quantized_lm_head is None
    assert "no accepted" in policy.reason


def test_failed_quality_gate_uses_exact_fallback():
    policy = P.select_qwen_policy(caps(9, 0), SIGNATURE, PROFILES)
    assert policy.profile == "fallback" and not policy.w8a16_layers


def test_model_signature_mismatch_uses_exact_fallback():
    policy = P.select_qwen_policy(caps(8, 9), P.ModelSignature(32, 1024, 16, 8, 128), PROFILES)
    assert not policy.calibrated and not policy.direct_attention_layers
    assert "signature" in policy.reason


def test_sm100_row_selects_quantized_layers():
    policy = P.select_qwen_policy(caps(10, 0), SIGNATURE, PROFILES)
    assert policy.calibrated and policy.profile == "b200"
    assert policy.layer_format(0) == "w8_row" and policy.layer_format(19) == "w8_row"
    assert policy.layer_format(20) == "w4_asym" and policy.layer_format(27) == "w4_asym"
    assert policy.quantized_lm_head == "w8_row"


@pytest.mark.parametrize("patch, message", [
    ({"w8a16_layers": [28]}, "invalid layer index"),
    ({"w4a16_layers": [-1]}, "invalid layer index"),
    ({"w8a16_layers": [3], "w4a16_layers": [3]}, "both"),
    ({"quantized_lm_head": "fp8"}, "lm_head"),
    ({"block_size": 24}, "block/tile"),
    ({"attention_tile": 96}, "block/tile"),
])
def test_invalid_rows_raise(patch, message):
    profiles = json.loads(json.dumps(PROFILES))
    profiles["architectures"]["sm100"].update(patch)
    with pytest.raises(ValueError, match=message):
        P.select_qwen_policy(caps(10, 0), SIGNATURE, profiles)


def test_packaged_profile():
    profiles = json.loads(P.DEFAULT_PROFILES.read_text())
    policy = P.select_qwen_policy(caps(10, 0), SIGNATURE, profiles)
    assert policy.calibrated and policy.w8a16_layers == frozenset(range(28))
    assert policy.quantized_lm_head == "w8_row"
    # other architectures are not claimed by this package's profile
    assert P.select_qwen_policy(caps(8, 9), SIGNATURE, profiles).profile == "fallback"
