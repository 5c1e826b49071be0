"""Int8 tensor-core mode of the grouped launch (``GroupedLinear(mma="int8")``).

The weights go to ``tcgen05.mma.kind::i8`` unconverted; each activation row is
split by a digits pass into a power-of-two scale s and three int8 planes with
x = s (65536 h + 256 m + l).  Parity is the BASELINE gate against the
fp32-accumulated oracle (max-abs 2e-2 or one bf16 ulp, rel-Frobenius 5e-3),
plus the mode's own accuracy claims: activations within a factor 2^14 of the
row's largest are represented exactly (outputs within one bf16 rounding of the
bf16-MMA mode), other activations are off by at most s / 2.
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
pytestmark = pytest.mark.gpu

QWEN_SHAPES = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072)]


def make(m, n, k, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).bfloat16()
    return x, w


def quantize(w):
    p = kl.quantize_int8_rowwise(w.cuda())
    q, s = O.quantize_int8_rowwise(w.numpy())
    np.testing.assert_array_equal(p.data.cpu().numpy(), q)
    return p, q, s


def oracle(x, q, s):
    return O.linear_f32(x.float().numpy(), O.dequantize_int8_rowwise(q, s))


def run_group(problems, **kw):
    g = kl.GroupedLinear(problems, **kw)
    g.run()
    torch.cuda.synchronize()
    assert kl._native.device_status(torch.cuda.current_device()) == 0
    return g


@pytest.mark.parametrize("m", [1, 2, 8, 9, 16, 17, 33, 64, 100, 256])
def test_int8_mode_matches_oracle(m):
    """Every token-tile size (8, 16, 32, 64; several tiles at M = 100, 256)."""
    probs, refs = [], []
    for i, (n, k) in enumerate(QWEN_SHAPES + [(200, 256), (17, 1024)]):
        x, w = make(m, n, k, seed=700 + i)
        p, q, s = quantize(w)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
        refs.append(oracle(x, q, s))
    g = run_group(probs, mma="int8")
    assert g.mma == "int8"
    for (x, p, y), ref in zip(probs, refs):
        assert_matches_oracle(y, ref, what=f"int8 mode {tuple(p.data.shape)} m={m}")


@pytest.mark.parametrize("m", [1, 16, 64])
def test_int8_mode_swiglu(m):
    n, k = 6144, 1024
    probs, refs = [], []
    for i in range(3):
        x, w = make(m, n, k, seed=800 + i)
        p, q, s = quantize(w)
        probs.append((x.cuda(), p, torch.empty(m, n // 2, device="cuda", dtype=torch.bfloat16)))
        refs.append(O.swiglu(O.bf16_round(oracle(x, q, s))))
    run_group(probs, swiglu=True, mma="int8")
    for (_, _, y), ref in zip(probs, refs):
        assert_matches_oracle(y, ref, what=f"int8 mode swiglu m={m}")


def test_int8_mode_exact_rows_match_bf16_mode():
    """Activations within a factor 2^14 of each row's largest are represented
    exactly, so both modes compute the same sums up to f32 rounding: outputs
    agree within one bf16 rounding step."""
    m, n, k = 8, 4096, 1024
    gen = torch.Generator().manual_seed(5)
    mag = torch.rand(m, k, generator=gen) * 3.0 + 0.5          # |x| in [0.5, 3.5): ratio < 2^14
    sign = torch.where(torch.rand(m, k, generator=gen) < 0.5, -1.0, 1.0)
    x = (mag * sign).bfloat16().cuda()
    w = torch.randn(n, k, generator=gen) * 0.02
    p, q, s = quantize(w)
    y8 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    yb = torch.empty_like(y8)
    run_group([(x, p, y8)], mma="int8")
    run_group([(x, p, yb)], mma="bf16")
    a, b = y8.float(), yb.float()
    ulp = torch.exp2(torch.floor(torch.log2(torch.clamp(b.abs(), min=2.0 ** -126))) - 7)
    assert bool(((a - b).abs() <= ulp).all())
    assert_matches_oracle(y8, oracle(x.cpu(), q, s), what="exact rows")


def test_int8_mode_wide_dynamic_range():
    """A row with one huge activation: the small ones are rounded to the grid
    s = 2^(floor(log2 max) - 21); the error stays within sum_k |w| * s / 2."""
    m, n, k = 4, 1024, 2048
    x, w = make(m, n, k, seed=11)
    x[0, 7] = 3.0e5
    x[1, 100] = -1.0e-4          # tiny values among normal ones
    x[2, :] = x[2, :] * 1e-30    # a row of tiny values (its own scale)
    x = x.bfloat16()
    p, q, s = quantize(w)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    run_group([(x.cuda(), p, y)], mma="int8")
    ref = oracle(x, q, s)
    deq = O.dequantize_int8_rowwise(q, s).astype(np.float64)
    xa = x.float().numpy().astype(np.float64)
    for t in range(m):
        amax = np.abs(xa[t]).max()
        grid = 2.0 ** (np.floor(np.log2(amax)) - 21)
        bound = np.abs(deq).sum(axis=1) * grid / 2 + np.abs(ref[t]) * 2.0 ** -8 + 1e-30
        err = np.abs(y[t].float().cpu().numpy() - ref[t])
        assert (err <= bound).all(), f"row {t}: worst {float((err - bound).max()):.3g} over the bound"


def test_int8_mode_zero_and_nonfinite_rows():
    m, n, k = 3, 1024, 1024
    x, w = make(m, n, k, seed=12)
    x[0].zero_()
    x[1, 5] = float("inf")
    p, q, s = quantize(w)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    run_group([(x.cuda(), p, y)], mma="int8")
    assert bool((y[0] == 0).all())
    assert bool(torch.isnan(y[1]).all())
    assert_matches_oracle(y[2:], oracle(x[2:], q, s), what="finite row beside non-finite ones")


def test_int8_mode_graph_replay_and_new_inputs():
    m = 8
    probs = []
    for i, (n, k) in enumerate(QWEN_SHAPES):
        x, w = make(m, n, k, seed=900 + i)
        p, _, _ = quantize(w)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
    g = run_group(probs, mma="int8")
    first = [y.clone() for _, _, y in probs]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g.run(pdl=True)
        g.run(pdl=True)
    for _, _, y in probs:
        y.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for a, (_, _, y) in zip(first, probs):
        assert torch.equal(a, y)
    for x, _, _ in probs:
        x.normal_()
    graph.replay()
    torch.cuda.synchronize()
    # an eager launch over the same problems (same partition) gives the same bits
    refs = [torch.empty_like(y) for _, _, y in probs]
    run_group([(x, p, r) for (x, p, _), r in zip(probs, refs)], mma="int8")
    for r, (_, _, y) in zip(refs, probs):
        assert torch.equal(r, y)


def test_int8_mode_rejects_other_formats():
    """The int8 mode takes int8 row weights and asymmetric 4-bit group-128
    weights with bf16 activations; the symmetric 4-bit format and f16
    activations are rejected."""
    x, w = make(1, 256, 256, seed=1)
    p = kl.quantize_int4(w.cuda(), 128)
    with pytest.raises(Exception):
        kl.GroupedLinear([(x.cuda(), p, torch.empty(1, 256, device="cuda", dtype=torch.bfloat16))], mma="int8")
    p8, _, _ = quantize(w)
    with pytest.raises(Exception):
        kl.GroupedLinear([(x.half().cuda(), p8, torch.empty(1, 256, device="cuda", dtype=torch.half))], mma="int8")
