"""Mirror of the reference's learning/10_cuda_decode/test_cuda_decode.py against
the B200 ``project`` op, plus the per-row (BASELINE) weight format."""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()


def test_calibration_cpu():
    torch.manual_seed(1)
    w, x = torch.randn(13, 128), torch.randn(8, 128)
    base = kl.quantize_int8(w, x, alphas=(0.,))
    calibrated = kl.quantize_int8(w, x)
    assert calibrated.calibration_mse <= base.calibration_mse
    assert calibrated.data.dtype == torch.int8
    zero = kl.quantize_int8(torch.zeros_like(w), x)
    assert torch.count_nonzero(kl.dequantize_int8(zero)) == 0
    with pytest.raises(ValueError):
        kl.quantize_int8(w[:, :127], x[:, :127])


def test_calibration_matches_reference_bits(golden):
    """The product quantiser is the reference's algorithm: identical packed bytes."""
    for name in ("cal_a", "cal_b", "cal_b_g64"):
        alphas = tuple(float(a) for a in golden[f"{name}_alphas"])
        p = kl.quantize_int8(torch.from_numpy(golden[f"{name}_w"]), torch.from_numpy(golden[f"{name}_x"]),
                             group_size=int(golden[f"{name}_group"]), alphas=alphas)
        np.testing.assert_array_equal(p.data.numpy(), golden[f"{name}_data"])
        np.testing.assert_array_equal(p.scales.numpy(), golden[f"{name}_scales"])
        np.testing.assert_array_equal(p.inverse.numpy(), golden[f"{name}_inverse"])
        assert p.alpha == float(golden[f"{name}_alpha"])


@pytest.mark.gpu
@pytest.mark.parametrize('warps,persistent', [(1, False), (4, False), (8, False), (4, True)])
@pytest.mark.parametrize('quant', [False, True])
@pytest.mark.parametrize('swiglu', [False, True])
def test_projection(warps, persistent, quant, swiglu):
    torch.manual_seed(42)
    torch.backends.cuda.matmul.allow_tf32 = False
    x = torch.randn(256, device='cuda', dtype=torch.bfloat16)
    w = torch.randn(34, 256, device='cuda', dtype=torch.bfloat16)
    packed = kl.quantize_int8(w, torch.randn(8, 256, device='cuda')) if quant else w
    restored = kl.dequantize_int8(packed) if quant else w.float()
    expected = (restored @ x.float()).bfloat16()
    if swiglu:
        a, b = expected.chunk(2)
        expected = torch.nn.functional.silu(a) * b
    actual = kl.project(x, packed, warps=warps, persistent=persistent, swiglu=swiglu)
    torch.testing.assert_close(actual, expected, rtol=.02, atol=.02)


@pytest.mark.gpu
def test_projection_golden(golden):
    """The reference's own expected outputs for its test inputs (bf16 weights and
    the calibrated int8 format)."""
    g = golden
    x = torch.from_numpy(g["proj_x"]).bfloat16().cuda()
    packed = kl.CalibratedInt8(torch.from_numpy(g["proj_data"]).cuda(), torch.from_numpy(g["proj_scales"]).cuda(),
                               torch.from_numpy(g["proj_inverse"]).cuda(), 128, float(g["proj_alpha"]), 0.0)
    y = kl.project(x, packed)
    assert_matches_oracle(y, g["proj_expected"], what="int8")
    ys = kl.project(x, packed, swiglu=True)
    assert_matches_oracle(ys, g["proj_expected_swiglu"], what="int8 swiglu")
    w = torch.from_numpy(g["proj_w"]).bfloat16().cuda()
    assert_matches_oracle(kl.project(x, w), g["proj_expected_bf16w"], what="bf16")


@pytest.mark.gpu
def test_tail_stream_and_reject():
    x = torch.randn(7, device='cuda', dtype=torch.bfloat16)
    w = torch.randn(33, 7, device='cuda', dtype=torch.bfloat16)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        y = kl.project(x, w, warps=1)
    torch.cuda.current_stream().wait_stream(stream)
    torch.testing.assert_close(y, (w.float() @ x.float()).bfloat16(), rtol=.02, atol=.01)
    with pytest.raises(RuntimeError):
        kl.project(x, w, swiglu=True)
    with pytest.raises(RuntimeError):
        kl.project(x, w, warps=2)


@pytest.mark.gpu
@pytest.mark.parametrize("swiglu", [False, True])
def test_project_rowwise_format(swiglu):
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=gen) * 0.02
    x = torch.randn(1024, generator=gen).bfloat16()
    q, s = O.quantize_int8_rowwise(w.numpy())
    packed = kl.RowwiseInt8(torch.from_numpy(q).cuda(), torch.from_numpy(O.bf16_bits(s).view(np.int16)).view(torch.bfloat16).cuda())
    y = kl.project(x.cuda(), packed, swiglu=swiglu)
    ref = O.linear_f32(x.float().numpy()[None], O.dequantize_int8_rowwise(q, s))[0]
    if swiglu:
        ref = O.swiglu(O.bf16_round(ref))
    assert_matches_oracle(y, ref, what="rowwise project")


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["cal_a", "cal_a_rtn", "cal_b", "cal_b_g64"])
def test_calibrated_dequantize_on_gpu_matches_reference_bits(golden, case):
    """kl_dequantize(KL_W8_GROUP) reproduces the reference's dequantize_int8
    (activation_int8.py:63-64, f32 q * s * inverse in that order) bit for bit
    on the weights the reference itself calibrated."""
    w = kl.CalibratedInt8(torch.from_numpy(golden[f"{case}_data"]).cuda(),
                          torch.from_numpy(golden[f"{case}_scales"]).cuda(),
                          torch.from_numpy(golden[f"{case}_inverse"]).cuda(),
                          int(golden[f"{case}_group"]), float(golden[f"{case}_alpha"]), float(golden[f"{case}_mse"]))
    got = kl.dequantize_native(w).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"{case}_deq"].view(np.uint32))
