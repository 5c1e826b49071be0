"""Qwen RMSNorm and the fused residual-add + RMSNorm
(reference ``learning/03_rmsnorm/qwen_rmsnorm.py``, tests in
``learning/03_rmsnorm/test_qwen_rmsnorm.py``): the oracle against vectors made by
the reference's own eager functions, then the CUDA kernels against both.
Tolerances are the reference test's, per dtype; the residual stream is exact."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import load_kl

HERE = Path(__file__).resolve().parent
GOLD = np.load(HERE / "golden" / "rmsnorm_vectors.npz")
TOL = {"f32": (2e-5, 2e-6), "f16": (2e-3, 2e-3), "bf16": (2e-2, 2e-2)}
TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def decode(a, dtype):
    if dtype == "f32":
        return a.astype(np.float32)
    if dtype == "f16":
        return a.view(np.float16).astype(np.float32)
    return O.bf16_to_f32(a)


def cases():
    keys = sorted({k.rsplit("_", 1)[0] for k in GOLD.files})
    return [(k, k.split("_")[0]) for k in keys]


def load_case(key, dtype):
    return {n: decode(GOLD[f"{key}_{n}"], dtype) for n in ("x", "r", "w", "y", "ry", "rc")}


@pytest.mark.parametrize("key,dtype", cases())
def test_oracle_matches_reference_vectors(key, dtype):
    c = load_case(key, dtype)
    rtol, atol = TOL[dtype]
    y = O.qwen_rmsnorm(c["x"], c["w"], dtype=dtype)
    np.testing.assert_allclose(y, c["y"], rtol=rtol, atol=atol)
    ry, rc = O.qwen_residual_rmsnorm(c["x"], c["r"], c["w"], dtype=dtype)
    np.testing.assert_array_equal(rc, c["rc"])
    np.testing.assert_allclose(ry, c["ry"], rtol=rtol, atol=atol)
    if dtype != "f32":
        # 16-bit outputs are pinned closely, not just within tolerance: nearly every
        # element is the reference's own (f32 differs in the last bits with the sum order)
        assert np.mean(y == c["y"]) >= 0.99 and np.mean(ry == c["ry"]) >= 0.99


def test_cases_cover_the_reference_tests():
    keys = {k for k, _ in cases()}
    for dt in TORCH:
        for shape in ("1x128", "33x128", "1x1024", "17x1024", "3x127"):
            assert f"{dt}_{shape}_s2" in keys


gpu = pytest.mark.gpu


def cuda(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(TORCH[dtype]).cuda()


@gpu
@pytest.mark.parametrize("key,dtype", cases())
def test_kernel_matches_reference_vectors(key, dtype):
    kl = load_kl()
    c = load_case(key, dtype)
    rtol, atol = TOL[dtype]
    x, r, w = cuda(c["x"], dtype), cuda(c["r"], dtype), cuda(c["w"], dtype)
    with torch.inference_mode():
        y = kl.qwen_rmsnorm(x, w)
        ry, rc = kl.qwen_residual_rmsnorm(x, r, w)
    np.testing.assert_allclose(y.float().cpu().numpy(), c["y"], rtol=rtol, atol=atol)
    np.testing.assert_array_equal(rc.float().cpu().numpy(), c["rc"])
    np.testing.assert_allclose(ry.float().cpu().numpy(), c["ry"], rtol=rtol, atol=atol)


def random_case(rows, n, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, n, generator=g) * scale).to(TORCH[dtype])
    r = torch.randn(rows, n, generator=g).to(TORCH[dtype])
    w = torch.randn(n, generator=g).to(TORCH[dtype])
    return x, r, w


@gpu
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rows,n", [(64, 2048), (5, 4096), (3, 8192), (2, 16384), (300, 1024), (9, 1000)])
@pytest.mark.parametrize("precise", [False, True])
def test_widths_and_math_modes(dtype, rows, n, precise):
    kl = load_kl()
    x, r, w = random_case(rows, n, dtype, seed=rows + n)
    with torch.inference_mode():
        ry, rc = kl.qwen_residual_rmsnorm(x.cuda(), r.cuda(), w.cuda(), precise_math=precise)
    ey, ec = O.qwen_residual_rmsnorm(x.float().numpy(), r.float().numpy(), w.float().numpy(), dtype=dtype)
    np.testing.assert_array_equal(rc.float().cpu().numpy(), ec)
    rtol, atol = TOL[dtype]
    np.testing.assert_allclose(ry.float().cpu().numpy(), ey, rtol=rtol, atol=atol)


@gpu
def test_unaligned_buffers_take_the_element_path():
    kl = load_kl()
    x, r, w = random_case(7, 1024, "bf16", seed=5)
    xb = torch.zeros(7 * 1024 + 1, dtype=torch.bfloat16, device="cuda")
    xs = xb[1:].view(7, 1024)                       # 2-byte aligned
    xs.copy_(x.cuda())
    with torch.inference_mode():
        y = kl.qwen_rmsnorm(xs, w.cuda())
    np.testing.assert_allclose(y.float().cpu().numpy(), O.qwen_rmsnorm(x.float().numpy(), w.float().numpy()),
                               rtol=2e-2, atol=2e-2)


@gpu
def test_prefill_rows_are_independent():
    """A full prefill block (8192 x 1024): sampled rows against the oracle, and
    the same rows normalised alone give the same bits."""
    kl = load_kl()
    x, r, w = random_case(8192, 1024, "bf16", seed=11)
    xc, rc_, wc = x.cuda(), r.cuda(), w.cuda()
    with torch.inference_mode():
        ry, rcs = kl.qwen_residual_rmsnorm(xc, rc_, wc)
        rows = [0, 1, 4095, 8191]
        alone, _ = kl.qwen_residual_rmsnorm(xc[rows].contiguous(), rc_[rows].contiguous(), wc)
    torch.testing.assert_close(alone, ry[rows], rtol=0, atol=0)
    ey, ec = O.qwen_residual_rmsnorm(x[rows].float().numpy(), r[rows].float().numpy(), w.float().numpy())
    np.testing.assert_array_equal(rcs[rows].float().cpu().numpy(), ec)
    np.testing.assert_allclose(ry[rows].float().cpu().numpy(), ey, rtol=2e-2, atol=2e-2)


@gpu
def test_reference_argument_errors():
    kl = load_kl()
    with pytest.raises(ValueError, match="contiguous"):
        kl.qwen_rmsnorm(torch.randn(128, 4, device="cuda").T, torch.ones(128, device="cuda"))
    with pytest.raises(ValueError, match="num_warps"):
        kl.qwen_rmsnorm(torch.randn(2, 128, device="cuda"), torch.ones(128, device="cuda"), num_warps=3)
    with pytest.raises(ValueError, match="dtype"):
        kl.qwen_rmsnorm(torch.randn(2, 128, device="cuda"), torch.ones(128, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="residual"):
        kl.qwen_residual_rmsnorm(torch.randn(2, 128, device="cuda"), torch.randn(3, 128, device="cuda"),
                                 torch.ones(128, device="cuda"))
    x = torch.empty(0, 128, device="cuda")
    assert kl.qwen_rmsnorm(x, torch.ones(128, device="cuda")).shape == x.shape
    assert kl.rmsnorm.triton_qwen_rmsnorm is kl.qwen_rmsnorm


def test_c_abi_rejects_bad_arguments_without_a_gpu():
    kl = load_kl()
    N = kl._native
    lib = N.lib()
    fake = 16
    assert lib.kl_rmsnorm(fake, None, fake, N.KL_DT_BF16, 1, 0, 1e-6, 0, fake, None, None) == N.KL_ERR_INVALID
    assert lib.kl_rmsnorm(fake, None, fake, N.KL_DT_BF16, 1, 16385, 1e-6, 0, fake, None, None) == N.KL_ERR_INVALID
    assert lib.kl_rmsnorm(fake, fake, fake, N.KL_DT_BF16, 1, 128, 1e-6, 0, fake, None, None) == N.KL_ERR_INVALID
    assert lib.kl_rmsnorm(fake, None, fake, 7, 1, 128, 1e-6, 0, fake, None, None) == N.KL_ERR_INVALID
    assert lib.kl_rmsnorm(fake, None, fake, N.KL_DT_BF16, 1, 128, 0.0, 0, fake, None, None) == N.KL_ERR_INVALID
    assert lib.kl_rmsnorm(fake, None, fake, N.KL_DT_BF16, 0, 128, 1e-6, 0, fake, None, None) == N.KL_OK
