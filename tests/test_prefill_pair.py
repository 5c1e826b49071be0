"""Edge cases of the CTA-pair prefill kernel (int8 row scale, M >= 256, K a
multiple of 64) against the oracle: ragged weight rows and tokens around the
256 x 192 pair tile, the transposed output layout, f16 activations, SwiGLU with
ragged gate/up widths, outputs that cannot take 16-byte stores, and the K that
falls back to the stream-K kernel."""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
N = kl._native
pytestmark = pytest.mark.gpu


def make(m, n, k, seed, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).to(dtype)
    p = kl.quantize_int8_rowwise(w.cuda())
    q, s = O.quantize_int8_rowwise(w.numpy())
    np.testing.assert_array_equal(p.data.cpu().numpy(), q)
    return x, p, q, s


def ref(x, q, s):
    return O.linear_f32(x.float().numpy(), O.dequantize_int8_rowwise(q, s))


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (257, 1000, 1024), (383, 1032, 640), (384, 4096, 1024),
                                   (1000, 520, 2048), (448, 128, 192)])
def test_ragged_tiles(m, n, k):
    x, p, q, s = make(m, n, k, seed=m + n)
    assert N.describe_plan(m, n, k, N.KL_W8_ROW)["kernel"] == 3
    assert_matches_oracle(kl.quant_linear(x.cuda(), p), ref(x, q, s), what=f"pair m={m} n={n} k={k}")


@pytest.mark.parametrize("m", [256, 700])
def test_transposed_output(m):
    x, p, q, s = make(m, 2048, 1024, seed=5)
    yt = kl.quant_linear(x.cuda(), p, transposed=True)
    assert yt.shape == (2048, m)
    assert_matches_oracle(yt.T, ref(x, q, s), what=f"pair transposed m={m}")


def test_f16_activations():
    x, p, q, s = make(512, 1024, 1024, seed=6, dtype=torch.float16)
    y = kl.quant_linear(x.cuda(), p)
    assert y.dtype == torch.float16
    r = ref(x, q, s)
    err = np.abs(y.float().cpu().numpy() - r)
    assert err.max() <= 2e-2 and np.linalg.norm(y.float().cpu().numpy() - r) / np.linalg.norm(r) <= 5e-3


@pytest.mark.parametrize("m,n", [(256, 6144), (300, 200), (600, 1000)])
def test_swiglu_ragged(m, n):
    x, p, q, s = make(m, n, 1024, seed=m * 3 + n)
    y = kl.quant_linear(x.cuda(), p, swiglu=True)
    assert y.shape == (m, n // 2)
    assert_matches_oracle(y, O.swiglu(O.bf16_round(ref(x, q, s))), what=f"pair swiglu m={m} n={n}")


def test_unaligned_output_uses_element_stores():
    """An output row stride that is not a multiple of 8 elements cannot take 16-byte stores."""
    m, n, k = 512, 1000, 512
    x, p, q, s = make(m, n, k, seed=9)
    big = torch.zeros(m * (n + 4), device="cuda", dtype=torch.bfloat16)
    y = big[2: 2 + m * n].view(m, n)                       # 4-byte aligned base
    kl.quant_linear(x.cuda(), p, out=y)
    assert_matches_oracle(y, ref(x, q, s), what="pair unaligned out")
    assert torch.count_nonzero(big[:2]) == 0 and torch.count_nonzero(big[2 + m * n:]) == 0


def test_k_not_multiple_of_64_uses_stream_k():
    m, n, k = 512, 1024, 1040
    x, p, q, s = make(m, n, k, seed=10)
    assert N.describe_plan(m, n, k, N.KL_W8_ROW)["kernel"] == 2
    assert_matches_oracle(kl.quant_linear(x.cuda(), p), ref(x, q, s), what="k=1040 fallback")


def test_repeated_calls_deterministic():
    x, p, q, s = make(2048, 3072, 1024, seed=12)
    xc = x.cuda()
    a = kl.quant_linear(xc, p)
    b = kl.quant_linear(xc, p)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    assert N.device_status(torch.cuda.current_device()) == 0


def test_pdl_chain_reads_previous_output():
    """With programmatic dependent launch the second GEMM starts while the first
    runs; its token loads must still see the first GEMM's finished output."""
    m, n1, k = 1024, 2048, 1024
    x, p1, q1, s1 = make(m, n1, k, seed=31)
    _, p2, q2, s2 = make(m, 1024, n1, seed=32)
    xc = x.cuda()
    for _ in range(3):
        y1 = kl.quant_linear(xc, p1, pdl=True)
        y2 = kl.quant_linear(y1, p2, pdl=True)
    torch.cuda.synchronize()
    assert_matches_oracle(y1, ref(x, q1, s1), what="pdl first")
    assert_matches_oracle(y2, ref(y1.cpu(), q2, s2), what="pdl second")


# ---- grouped launches on the pair kernel (every problem M >= 256, K % 64 == 0)

def _grouped(problems, swiglu=False):
    g = kl.GroupedLinear(problems, swiglu=swiglu)
    g.run()
    torch.cuda.synchronize()
    assert N.device_status(torch.cuda.current_device()) == 0
    return g


@pytest.mark.parametrize("m", [256, 300, 512])
def test_grouped_pair_layer(m):
    """A Qwen3 layer's four GEMMs plus ragged shapes in one pair launch."""
    shapes = [(4096, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (520, 640), (130, 192)]
    probs, refs = [], []
    for i, (n, k) in enumerate(shapes):
        x, p, q, s = make(m, n, k, seed=1000 + i + m)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
        refs.append(ref(x, q, s))
    _grouped(probs)
    for (_, p, y), r in zip(probs, refs):
        assert_matches_oracle(y, r, what=f"grouped pair {tuple(p.data.shape)} m={m}")


def test_grouped_pair_swiglu_and_f16():
    m = 320
    probs, refs = [], []
    for i in range(2):
        x, p, q, s = make(m, 6144, 1024, seed=1100 + i)
        probs.append((x.cuda(), p, torch.empty(m, 3072, device="cuda", dtype=torch.bfloat16)))
        refs.append(O.swiglu(O.bf16_round(ref(x, q, s))))
    _grouped(probs, swiglu=True)
    for (_, _, y), r in zip(probs, refs):
        assert_matches_oracle(y, r, what="grouped pair swiglu")
    x, p, q, s = make(256, 1024, 1024, seed=1200, dtype=torch.float16)
    y = torch.empty(256, 1024, device="cuda", dtype=torch.float16)
    _grouped([(x.cuda(), p, y), (x.cuda(), p, torch.empty_like(y))])
    assert_matches_oracle(y, ref(x, q, s), what="grouped pair f16")


def test_grouped_pair_matches_single_calls_and_replays():
    """Whole-K tiles: the grouped launch gives the same bits as one call per
    problem, eagerly and when replayed from a CUDA graph."""
    m = 512
    probs = []
    for i, (n, k) in enumerate([(4096, 1024), (1024, 2048), (1024, 3072)]):
        x, p, _, _ = make(m, n, k, seed=1300 + i)
        probs.append((x.cuda(), p, torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
    g = _grouped(probs)
    for x, p, y in probs:
        assert torch.equal(kl.quant_linear(x, p), y)
    graph = torch.cuda.CUDAGraph()
    first = [y.clone() for _, _, y in probs]
    with torch.cuda.graph(graph):
        g.run(pdl=True)
    for _, _, y in probs:
        y.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for a, (_, _, y) in zip(first, probs):
        assert torch.equal(a, y)


def test_grouped_mixed_m_stays_on_stream_k():
    """A group with any problem under 256 tokens keeps the stream-K kernel."""
    probs, refs = [], []
    for i, m in enumerate([256, 64]):
        x, p, q, s = make(m, 1024, 1024, seed=1400 + i)
        probs.append((x.cuda(), p, torch.empty(m, 1024, device="cuda", dtype=torch.bfloat16)))
        refs.append(ref(x, q, s))
    _grouped(probs)
    for (_, _, y), r in zip(probs, refs):
        assert_matches_oracle(y, r, what="mixed-m group")
