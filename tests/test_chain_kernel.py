"""Parity of the single-tile cluster kernel (the decode linear for dependent
chains, ``kl_describe_plan`` kernel 4) against the oracle and against the
persistent stream-K kernel it replaces for one decode-size linear.

Same gate as every W8A16 test: outputs within max-abs 2e-2 (one bf16 ulp where
larger) and relative Frobenius 5e-3 of the fp32-accumulated reference
(dequantise-then-matmul, ``decode_stage2_benchmark.py:55`` of the reference).
"""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
N = kl._native
pytestmark = pytest.mark.gpu

QWEN = {"qkv": (4096, 1024), "o": (1024, 2048), "gate_up": (6144, 1024), "down": (1024, 3072)}


def make(m, n, k, seed=0, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).to(dtype)
    p = kl.quantize_int8_rowwise(w.cuda())
    return x, p, p.data.cpu().numpy(), p.scales.float().cpu().numpy()


def oracle(x, q, s, swiglu=False):
    y = O.linear_f32(x.float().numpy(), O.dequantize_int8_rowwise(q, s))
    return O.swiglu(O.bf16_round(y)) if swiglu else y


def kernel_of(m, n, k, swiglu=False, flags=N.KL_FLAG_FORCE_TC):
    return N.describe_plan(m, n, k, N.KL_W8_ROW, swiglu=swiglu, flags=flags,
                           sm_count=torch.cuda.get_device_properties(0).multi_processor_count)["kernel"]


@pytest.mark.parametrize("m", [1, 2, 5, 8, 16, 17, 31, 32, 33, 48, 64])
@pytest.mark.parametrize("name", list(QWEN))
def test_config1_shapes(m, name):
    n, k = QWEN[name]
    sw = name == "gate_up"
    assert kernel_of(m, n, k, sw) == 4
    x, p, q, s = make(m, n, k, seed=m)
    ref = oracle(x, q, s, sw)
    y = kl.quant_linear(x.cuda(), p, swiglu=sw, path="tc")
    assert_matches_oracle(y, ref, what=f"{name} m={m} chain")
    # the persistent kernel on the same inputs meets the same gate
    yp = kl.quant_linear(x.cuda(), p, swiglu=sw, path="persistent")
    assert_matches_oracle(yp, ref, what=f"{name} m={m} persistent")


@pytest.mark.parametrize("m,n,k,sw", [
    (1, 17, 128, False),        # one K block, one partial tile, cluster of 1
    (3, 129, 1040, False),      # K not a multiple of 128: zero-filled last block
    (7, 1000, 1040, True),      # SwiGLU with a partial last gate tile
    (9, 200, 256, True),        # two K blocks, one CTA
    (64, 3072, 3072, False),    # Llama o: three blocks per CTA
    (33, 384, 4096, False),     # clusters of 8 with four blocks per CTA
])
def test_ragged_shapes(m, n, k, sw):
    assert kernel_of(m, n, k, sw) == 4
    x, p, q, s = make(m, n, k, seed=n + k)
    assert_matches_oracle(kl.quant_linear(x.cuda(), p, swiglu=sw, path="tc"), oracle(x, q, s, sw),
                          what=f"{m}x{n}x{k} sw={sw}")


def test_f16_and_transposed():
    m, n, k = 12, 4096, 1024
    x, p, q, s = make(m, n, k, seed=3, dtype=torch.float16)
    ref = oracle(x, q, s)
    y = kl.quant_linear(x.cuda(), p)
    assert y.dtype == torch.float16
    assert_matches_oracle(y, ref, what="f16")
    yt = kl.quant_linear(x.cuda(), p, transposed=True)
    assert yt.shape == (n, m)
    torch.testing.assert_close(yt.T, y, rtol=0, atol=0)


def test_deterministic():
    """K-split partial sums are added in cluster-rank order: bit-identical runs."""
    x, p, _, _ = make(40, 1024, 3072, seed=9)
    xc = x.cuda()
    a = kl.quant_linear(xc, p)
    for _ in range(3):
        torch.testing.assert_close(kl.quant_linear(xc, p), a, rtol=0, atol=0)


def test_dependent_chain_in_graph():
    """A model-forward pattern: every linear reads the previous one's output,
    all launched with programmatic dependent launch and captured in one CUDA
    graph; the replay equals eager execution and the oracle run in sequence."""
    m = 4
    dims = [1024, 4096, 1024, 3072, 1024, 2048, 1024]
    layers = [make(1, dims[i + 1], dims[i], seed=20 + i) for i in range(len(dims) - 1)]
    gen = torch.Generator().manual_seed(1)
    x0 = (torch.randn(m, dims[0], generator=gen)).bfloat16()
    bufs = [x0.cuda()] + [torch.empty(m, d, dtype=torch.bfloat16, device="cuda") for d in dims[1:]]

    def forward():
        for i, (_, p, _, _) in enumerate(layers):
            kl.quant_linear(bufs[i], p, out=bufs[i + 1], pdl=True)

    forward()
    torch.cuda.synchronize()
    eager = bufs[-1].clone()
    # oracle in sequence, each step rounded to bf16 like the kernel output
    h = x0.float().numpy()
    for i, (_, _, q, s) in enumerate(layers):
        ref = O.linear_f32(h, O.dequantize_int8_rowwise(q, s))
        assert_matches_oracle(bufs[i + 1], ref, what=f"chain step {i}")
        h = O.bf16_round(bufs[i + 1].float().cpu().numpy())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        forward()
    bufs[-1].zero_()
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(bufs[-1], eager, rtol=0, atol=0)


def test_persistent_flag_and_large_problems():
    """KL_FLAG_PERSISTENT keeps the stream-K kernel; problems too large for one
    cluster per tile (the 151,936-row lm_head) stay on it automatically."""
    assert kernel_of(1, 4096, 1024, flags=N.KL_FLAG_PERSISTENT) == 2
    assert kernel_of(1, 151936, 1024) == 2
    assert kernel_of(65, 4096, 1024) == 2
    assert kernel_of(1, 4096, 1024, flags=0) == 5                 # one token: CUDA-core chain GEMV
    assert N.device_status(0) == 0


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("name", list(QWEN))
def test_cuda_core_chain_gemv(m, name):
    """One or two tokens: the CUDA-core chain GEMV (kernel 5), full rows per CTA."""
    n, k = QWEN[name]
    sw = name == "gate_up"
    assert kernel_of(m, n, k, sw, flags=0) == 5
    x, p, q, s = make(m, n, k, seed=40 + m)
    ref = oracle(x, q, s, sw)
    assert_matches_oracle(kl.quant_linear(x.cuda(), p, swiglu=sw), ref, what=f"{name} m={m} gemv chain")
    yt = kl.quant_linear(x.cuda(), p, swiglu=sw, transposed=True)
    assert_matches_oracle(yt.T, ref, what=f"{name} m={m} gemv chain transposed")


@pytest.mark.parametrize("m,n,k,sw,dtype", [(1, 17, 128, False, torch.bfloat16), (2, 1000, 1040, True, torch.bfloat16),
                                            (1, 3072, 3072, False, torch.float16), (2, 4736, 256, False, torch.float16)])
def test_cuda_core_chain_gemv_ragged(m, n, k, sw, dtype):
    assert kernel_of(m, n, k, sw, flags=0) == 5
    x, p, q, s = make(m, n, k, seed=n, dtype=dtype)
    y = kl.quant_linear(x.cuda(), p, swiglu=sw)
    assert y.dtype == dtype
    assert_matches_oracle(y, oracle(x, q, s, sw), what=f"{m}x{n}x{k}")


def make_w4(m, n, k, fmt, group=128, seed=0, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).to(dtype)
    if fmt == "asym":
        p = kl.quantize_int4_asym(w.cuda(), group)
        deq = O.dequantize_int4_asym(p.data.cpu().numpy(), p.scales.float().cpu().numpy(),
                                     p.zeros.float().cpu().numpy(), group)
    else:
        p = kl.quantize_int4(w.cuda(), group)
        deq = O.dequantize_int4(p.data.cpu().numpy(), p.scales.cpu().numpy(), group)
    return x, p, deq


@pytest.mark.parametrize("fmt", ["asym", "sym"])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("name", list(QWEN))
def test_cuda_core_chain_gemv_w4(fmt, m, name):
    """4-bit weights, one or two tokens: the chain GEMV (kernel 5) with the
    group scale applied per 16-element chunk and the zero point folded into the
    exact integer conversion."""
    n, k = QWEN[name]
    sw = name == "gate_up"
    f = N.KL_W4_ASYM if fmt == "asym" else N.KL_W4_SYM
    assert N.describe_plan(m, n, k, f, swiglu=sw, sm_count=torch.cuda.get_device_properties(0).multi_processor_count)["kernel"] == 5
    x, p, deq = make_w4(m, n, k, fmt, seed=60 + m)
    ref = O.linear_f32(x.float().numpy(), deq)
    if sw:
        ref = O.swiglu(O.bf16_round(ref))
    y = kl.quant_linear(x.cuda(), p, swiglu=sw)
    assert_matches_oracle(y, ref, what=f"w4 {fmt} {name} m={m} gemv chain")
    yt = kl.quant_linear(x.cuda(), p, swiglu=sw, transposed=True)
    assert_matches_oracle(yt.T, ref, what=f"w4 {fmt} {name} m={m} transposed")
    # the persistent tcgen05 kernel on the same inputs meets the same gate
    yp = kl.quant_linear(x.cuda(), p, swiglu=sw, path="persistent")
    assert_matches_oracle(yp, ref, what=f"w4 {fmt} {name} m={m} persistent")


@pytest.mark.parametrize("fmt,m,n,k,group,dtype", [
    ("sym", 1, 17, 128, 32, torch.bfloat16),      # group 32: four groups per 128 columns
    ("sym", 2, 1000, 1088, 64, torch.float16),    # group 64, K not a multiple of 128
    ("asym", 1, 300, 4096, 128, torch.float16),
    ("asym", 2, 4733, 256, 128, torch.bfloat16),  # 32 rows per CTA, partial last CTA
])
def test_cuda_core_chain_gemv_w4_ragged(fmt, m, n, k, group, dtype):
    x, p, deq = make_w4(m, n, k, fmt, group=group, seed=n, dtype=dtype)
    y = kl.quant_linear(x.cuda(), p)
    assert y.dtype == dtype
    assert_matches_oracle(y, O.linear_f32(x.float().numpy(), deq), what=f"w4 {fmt} {m}x{n}x{k} g{group}")
    assert N.device_status(0) == 0


@pytest.mark.parametrize("m,n,k,sw,fmt", [
    (1, 6144, 1024, False, "w8"),     # gate_up without SwiGLU: 42 rows per CTA, 8 rows per warp
    (2, 6144, 1024, False, "w8"),
    (1, 5120, 3072, False, "w8"),     # Llama-3.2-3B fused QKV: 35 rows per CTA
    (1, 12288, 1024, True, "w8"),     # SwiGLU pair with 42 gate rows per CTA
    (1, 6144, 1024, False, "asym"),
    (2, 9472, 512, False, "sym"),     # 64 rows per CTA, the most the kernel takes
])
def test_cuda_core_chain_gemv_eight_rows_per_warp(m, n, k, sw, fmt):
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    f = {"w8": N.KL_W8_ROW, "asym": N.KL_W4_ASYM, "sym": N.KL_W4_SYM}[fmt]
    plan = N.describe_plan(m, n, k, f, swiglu=sw, sm_count=sm)
    assert plan["kernel"] == 5 and plan["stages"] == (8 if plan["tiles"] > 32 else 4)
    if fmt == "w8":
        x, p, q, s = make(m, n, k, seed=n + m)
        ref = oracle(x, q, s, sw)
    else:
        x, p, deq = make_w4(m, n, k, fmt, seed=n + m)
        ref = O.linear_f32(x.float().numpy(), deq)
    assert_matches_oracle(kl.quant_linear(x.cuda(), p, swiglu=sw), ref, what=f"{fmt} {m}x{n}x{k} sw={sw}")
    assert N.device_status(0) == 0
    # two-token SwiGLU above 32 rows per CTA stays on the tcgen05 chain kernel
    assert kernel_of(2, 12288, 1024, True, flags=0) == 4
