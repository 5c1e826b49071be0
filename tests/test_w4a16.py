"""Parity of the W4A16 linear (asymmetric int4, bf16 scale and
zero point per 128-group; and the reference's symmetric format)."""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
pytestmark = pytest.mark.gpu

QWEN = {"qkv": (4096, 1024), "o": (1024, 2048), "gate_up": (6144, 1024), "down": (1024, 3072),
        "lm_head": (151936, 1024)}


def make(m, n, k, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).bfloat16()
    return x, w


def quantize_asym(w, group=128):
    p = kl.quantize_int4_asym(w.cuda(), group)
    d, s, z = O.quantize_int4_asym(w.numpy(), group)
    np.testing.assert_array_equal(p.data.cpu().numpy(), d)
    np.testing.assert_array_equal(p.scales.float().cpu().numpy(), s)
    np.testing.assert_array_equal(p.zeros.float().cpu().numpy(), z)
    return p, d, s, z


@pytest.mark.parametrize("m", [1, 16])
@pytest.mark.parametrize("name", list(QWEN))
def test_config3_shapes(m, name):
    n, k = QWEN[name]
    x, w = make(m, n, k, seed=m + len(name))
    p, d, s, z = quantize_asym(w)
    y = kl.quant_linear(x.cuda(), p)
    rows = np.sort(np.random.default_rng(0).choice(n, min(n, 1024), replace=False))
    deq = O.dequantize_int4_asym(d[rows], s[rows], z[rows], 128)
    assert_matches_oracle(y[:, torch.from_numpy(rows).cuda()], O.linear_f32(x.float().numpy(), deq),
                          what=f"w4 {name} m={m}")


@pytest.mark.parametrize("m", [1, 3, 17, 64, 100, 300])
def test_w4_asym_tokens(m):
    x, w = make(m, 4096, 1024, seed=m)
    p, d, s, z = quantize_asym(w)
    ref = O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d, s, z, 128))
    assert_matches_oracle(kl.quant_linear(x.cuda(), p), ref, what=f"w4 tc m={m}")
    if m <= 4:
        assert_matches_oracle(kl.quant_linear(x.cuda(), p, path="simt"), ref, what=f"w4 simt m={m}")


def test_w4_dequant_bit_exact():
    _, w = make(1, 300, 512, seed=2)
    p, d, s, z = quantize_asym(w)
    torch.testing.assert_close(kl.dequantize_native(p).cpu(), torch.from_numpy(O.dequantize_int4_asym(d, s, z, 128)),
                               rtol=0, atol=0)


@pytest.mark.parametrize("m", [1, 16])
def test_w4_swiglu(m):
    x, w = make(m, 6144, 1024, seed=3)
    p, d, s, z = quantize_asym(w)
    ref = O.swiglu(O.bf16_round(O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d, s, z, 128))))
    assert_matches_oracle(kl.quant_linear(x.cuda(), p, swiglu=True), ref, what=f"w4 swiglu m={m}")


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("m", [1, 16])
def test_w4_symmetric_reference_format(group, m):
    x, w = make(m, 2048, 1024, seed=group)
    p = kl.quantize_int4(w.cuda(), group)
    d, s = O.quantize_int4(w.numpy(), group)
    np.testing.assert_array_equal(p.data.cpu().numpy(), d)
    np.testing.assert_array_equal(p.scales.cpu().numpy(), s)
    ref = O.linear_f32(x.float().numpy(), O.dequantize_int4(d, s, group))
    assert_matches_oracle(kl.quant_linear(x.cuda(), p), ref, what=f"w4 sym g={group} m={m}")


def test_w4_f16_activations():
    gen = torch.Generator().manual_seed(4)
    w = torch.randn(1024, 1024, generator=gen) * 0.02
    x = torch.randn(16, 1024, generator=gen).half()
    p, d, s, z = quantize_asym(w)
    ref = O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d, s, z, 128))
    y = kl.quant_linear(x.cuda(), p)
    assert y.dtype == torch.float16
    err = np.abs(y.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and np.linalg.norm(y.float().cpu().numpy() - ref) / np.linalg.norm(ref) <= 5e-3


@pytest.mark.parametrize("m", [1, 16])
def test_w4_grouped(m):
    probs, refs = [], []
    for i, (name, (n, k)) in enumerate(QWEN.items()):
        x, w = make(m, n, k, seed=50 + i)
        p, d, s, z = quantize_asym(w)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
        rows = np.sort(np.random.default_rng(i).choice(n, min(n, 512), replace=False))
        refs.append((rows, O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d[rows], s[rows], z[rows], 128))))
    kl.GroupedLinear(probs).run()
    torch.cuda.synchronize()
    for (_, p, y), (rows, ref) in zip(probs, refs):
        assert_matches_oracle(y[:, torch.from_numpy(rows).cuda()], ref, what=f"w4 grouped m={m}")


@pytest.mark.parametrize("mma", ["int8", "bf16"])
@pytest.mark.parametrize("m", [1, 5, 9, 16])
def test_w4_grouped_modes(m, mma):
    """Both tensor-core modes of the grouped 4-bit launch: int8 (q - z) against
    the activation digit planes (token tiles of 8 and 16) and bf16 (q - z)."""
    shapes = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (200, 256)]
    probs, refs = [], []
    for i, (n, k) in enumerate(shapes):
        x, w = make(m, n, k, seed=70 + i + m)
        p, d, s, z = quantize_asym(w)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
        refs.append(O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d, s, z, 128)))
    g = kl.GroupedLinear(probs, mma=mma)
    assert g.mma == mma
    g.run()
    torch.cuda.synchronize()
    assert kl._native.device_status(torch.cuda.current_device()) == 0
    for (_, p, y), ref in zip(probs, refs):
        assert_matches_oracle(y, ref, what=f"w4 grouped {mma} {tuple(p.data.shape)} m={m}")


def test_w4_grouped_int8_swiglu_and_replay():
    m, n, k = 16, 6144, 1024
    probs, refs = [], []
    for i in range(2):
        x, w = make(m, n, k, seed=90 + i)
        p, d, s, z = quantize_asym(w)
        probs.append((x.cuda(), p, torch.empty(m, n // 2, device="cuda", dtype=torch.bfloat16)))
        refs.append(O.swiglu(O.bf16_round(O.linear_f32(x.float().numpy(), O.dequantize_int4_asym(d, s, z, 128)))))
    g = kl.GroupedLinear(probs, swiglu=True, mma="int8")
    assert g.mma == "int8"
    g.run()
    torch.cuda.synchronize()
    for (_, _, y), ref in zip(probs, refs):
        assert_matches_oracle(y, ref, what="w4 int8 swiglu")
    first = [y.clone() for _, _, y in probs]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g.run(pdl=True)
    for _, _, y in probs:
        y.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for a, (_, _, y) in zip(first, probs):
        assert torch.equal(a, y)
