"""Pins the numpy oracle to the reference implementation's own outputs.

``tests/golden/reference_vectors.npz`` was produced by running the reference's
``activation_int8.py`` / ``quantization.py`` (``tests/golden/make_golden.py``).
Integer and byte outputs must match bit for bit.
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O


@pytest.mark.parametrize("name", ["cal_a", "cal_a_rtn", "cal_b", "cal_b_g64"])
def test_calibrated_int8_matches_reference(golden, name):
    g = golden
    alphas = tuple(float(a) for a in g[f"{name}_alphas"])
    r = O.quantize_int8(g[f"{name}_w"], g[f"{name}_x"], int(g[f"{name}_group"]), alphas)
    assert r["alpha"] == float(g[f"{name}_alpha"])
    np.testing.assert_array_equal(r["data"], g[f"{name}_data"])
    np.testing.assert_array_equal(r["scales"], g[f"{name}_scales"])
    # torch's vectorised sqrt (alpha 0.5) is not always correctly rounded; the
    # oracle uses IEEE sqrt, so a channel entry may differ by 1 ulp (its
    # reciprocal, the stored inverse, by up to 2); codes and scales are exact.
    np.testing.assert_array_max_ulp(r["inverse"], g[f"{name}_inverse"], maxulp=2)
    np.testing.assert_allclose(r["calibration_mse"], float(g[f"{name}_mse"]), rtol=1e-4)
    deq = O.dequantize_int8(g[f"{name}_data"], g[f"{name}_scales"], g[f"{name}_inverse"], int(g[f"{name}_group"]))
    np.testing.assert_array_equal(deq, g[f"{name}_deq"])


def test_zero_weights_dequantise_to_zero(golden):
    assert np.count_nonzero(golden["cal_zero_deq"]) == 0
    z = O.quantize_int8(np.zeros((13, 128), np.float32), np.random.default_rng(0).standard_normal((8, 128)))
    assert np.count_nonzero(O.dequantize_int8(z["data"], z["scales"], z["inverse"], 128)) == 0
    with pytest.raises(ValueError):
        O.quantize_int8(np.ones((13, 127), np.float32), np.ones((8, 127), np.float32))


@pytest.mark.parametrize("group", [32, 64, 128])
def test_int4_pack_matches_reference(golden, group):
    d, s = O.quantize_int4(golden[f"i4_rt{group}_w"], group, chunk_rows=2)
    np.testing.assert_array_equal(d, golden[f"i4_rt{group}_data"])
    np.testing.assert_array_equal(s, golden[f"i4_rt{group}_scales"])
    np.testing.assert_array_equal(O.dequantize_int4(d, s, group), golden[f"i4_rt{group}_w"])  # bit-exact round trip
    d, s = O.quantize_int4(golden[f"i4_err{group}_w"], group)
    np.testing.assert_array_equal(d, golden[f"i4_err{group}_data"])
    np.testing.assert_array_equal(s, golden[f"i4_err{group}_scales"])
    np.testing.assert_array_equal(O.dequantize_int4(d, s, group), golden[f"i4_err{group}_deq"])
    bound = np.repeat(s, group, axis=1) / 2 + 1e-6
    assert (np.abs(golden[f"i4_err{group}_w"] - O.dequantize_int4(d, s, group)) <= bound).all()


def test_int4_zero_group(golden):
    d, s = O.quantize_int4(np.zeros((2, 128), np.float32))
    np.testing.assert_array_equal(d, golden["i4_zero_data"])
    np.testing.assert_array_equal(s, golden["i4_zero_scales"])


def test_projection_oracle_matches_reference(golden):
    g = golden
    deq = O.dequantize_int8(g["proj_data"], g["proj_scales"], g["proj_inverse"], 128)
    y = O.linear(g["proj_x"][None], deq)[0]
    np.testing.assert_array_equal(y, g["proj_expected"])
    np.testing.assert_array_equal(O.swiglu(y), g["proj_expected_swiglu"])
    np.testing.assert_array_equal(O.linear(g["proj_x"][None], g["proj_w"])[0], g["proj_expected_bf16w"])


def test_swiglu_matches_torch_bf16(golden):
    e = O.swiglu(golden["swiglu_in"])
    np.testing.assert_array_equal(e, golden["swiglu_expected"])


def test_int4_head_and_topk(golden):
    g = golden
    logits = O.head_logits(g["i4_head_x"][None], O.dequantize_int4(g["i4_head_data"], g["i4_head_scales"], 128))[0]
    np.testing.assert_array_equal(logits, g["i4_head_logits"])
    for top in (1, 4, 8):
        v, i = O.topk_lowest_index(logits, top)
        np.testing.assert_array_equal(v, g[f"i4_head_top{top}_values"])
        np.testing.assert_array_equal(i, g[f"i4_head_top{top}_ids"])
    y = O.linear(g["i4_gemv_x"][None], O.dequantize_int4(g["i4_gemv_data"], g["i4_gemv_scales"], 128))[0]
    np.testing.assert_array_equal(y, g["i4_gemv_expected"])


def test_topk_tie_rule():
    v, i = O.topk_lowest_index(np.zeros(65, np.float32), 1)
    assert i[0] == 0


def _config0():
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=gen) * 0.02
    x = torch.randn(1, 1024, generator=gen).bfloat16()
    return x, w


def test_config0_against_reference(golden):
    """BASELINE config 0 through the reference quantiser (group = K, alpha 0)."""
    x, w = _config0()
    assert hashlib.sha256(w.numpy().tobytes()).hexdigest() == str(golden["cfg0_w_sha256"])
    r = O.quantize_int8(w.numpy(), x.float().numpy(), 1024, (0.0,))
    assert hashlib.sha256(r["data"].tobytes()).hexdigest() == str(golden["cfg0_data_sha256"])
    np.testing.assert_array_equal(r["scales"], golden["cfg0_scales"])
    np.testing.assert_array_equal(np.unique(r["inverse"]), golden["cfg0_inverse_unique"])
    y = O.linear_f32(x.float().numpy(), O.dequantize_int8(r["data"], r["scales"], r["inverse"], 1024))[0]
    # fp32 matmul order differs between numpy and torch: compare at bf16 granularity
    np.testing.assert_allclose(O.bf16_round(y), golden["cfg0_expected"], rtol=0, atol=2 ** -7)
    # BASELINE per-row format: the stored scale is the bf16 rounding of absmax/127
    q, s = O.quantize_int8_rowwise(w.numpy())
    np.testing.assert_array_equal(s, O.bf16_round(golden["cfg0_scales"][:, 0]))
    assert np.abs(q.astype(np.int32)).max() <= 127


def test_asym_int4_definition():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((9, 256)) * 0.02).astype(np.float32)
    d, s, z = O.quantize_int4_asym(w, 128)
    assert d.dtype == np.uint8 and d.shape == (9, 128)
    assert np.array_equal(s, O.bf16_round(s)) and np.array_equal(z, np.rint(z))
    assert (z >= 0).all() and (z <= 15).all()
    deq = O.dequantize_int4_asym(d, s, z, 128)
    # asymmetric RTN error bound: half a step, plus clamping of the range ends
    step = np.repeat(s, 128, axis=1)
    assert (np.abs(w - deq) <= step * 0.5 + np.abs(w) * 2 ** -7 + 1e-6).all()
