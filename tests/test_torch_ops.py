"""The registered operators ``torch.ops.kl_b200.*`` (``ops.py``): the role of the
reference's compiled extension op (``learning/10_cuda_decode/warp_gemv.cu:91``
loaded by ``cuda_decode.py:9-14``).  CPU: registration, schemas and FakeTensor
shape propagation.  GPU: eager results equal the Python API's, and the ops
work under CUDA-graph capture and ``torch.compile``."""
import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
N = kl._native


def test_ops_registered_with_schemas():
    for name in kl.ops.OPS:
        op = getattr(torch.ops.kl_b200, name)
        assert op.default._schema.name == f"kl_b200::{name}"
    # linear_out mutates its output argument only
    schema = torch.ops.kl_b200.linear_out.default._schema
    mutated = [a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write]
    assert mutated == ["out"]


@pytest.mark.parametrize("fmt,shape", [(N.KL_W8_ROW, (4096, 1024)), (N.KL_W4_ASYM, (6144, 512)),
                                       (N.KL_BF16_DENSE, (128, 1024))])
def test_fake_tensor_shapes(fmt, shape):
    n, kd = shape
    with FakeTensorMode():
        k = 1024
        x = torch.empty(7, k, dtype=torch.bfloat16, device="cuda")
        dt = torch.bfloat16 if fmt == N.KL_BF16_DENSE else (torch.uint8 if fmt == N.KL_W4_ASYM else torch.int8)
        d = torch.empty(n, kd, dtype=dt, device="cuda")
        s = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.kl_b200.linear(x, d, s, None, None, fmt, 128, False, False, 0)
        assert y.shape == (7, n) and y.dtype == torch.bfloat16 and y.device.type == "cuda"
        assert torch.ops.kl_b200.linear(x, d, s, None, None, fmt, 128, True, False, 0).shape == (7, n // 2)
        assert torch.ops.kl_b200.linear(x, d, s, None, None, fmt, 128, False, True, 0).shape == (n, 7)
        out = torch.empty(7, n, dtype=torch.bfloat16, device="cuda")
        assert torch.ops.kl_b200.linear_out(x, d, s, None, None, fmt, 128, False, False, 0, out) is None


def test_fake_tensor_reference_ops():
    with FakeTensorMode():
        x = torch.empty(1024, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(6144, 1024, dtype=torch.int8, device="cuda")
        sc = torch.empty(6144, 8, dtype=torch.float32, device="cuda")
        inv = torch.empty(1024, dtype=torch.float32, device="cuda")
        assert torch.ops.kl_b200.project(x, w, sc, inv, 128, 4, False, True).shape == (3072,)
        pk = torch.empty(151936, 512, dtype=torch.uint8, device="cuda")
        s4 = torch.empty(151936, 8, dtype=torch.float32, device="cuda")
        assert torch.ops.kl_b200.int4_gemv(x, pk, s4, 128, 32).shape == (151936,)
        v, i = torch.ops.kl_b200.int4_lm_head_topk(x, pk, s4, 128, 4, 32)
        assert v.shape == i.shape == (4,) and v.dtype == torch.float32 and i.dtype == torch.int64


@pytest.mark.gpu
def test_linear_op_eager_graph_and_compile():
    m, n, k = 8, 4096, 1024
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(n, k, generator=gen) * 0.02
    x = torch.randn(m, k, generator=gen).bfloat16().cuda()
    p = kl.quantize_int8_rowwise(w.cuda())
    ref = O.linear_f32(x.float().cpu().numpy(), O.dequantize_int8_rowwise(p.data.cpu().numpy(),
                                                                        p.scales.float().cpu().numpy()))
    y = torch.ops.kl_b200.linear(x, p.data, p.scales, None, None, N.KL_W8_ROW, k)
    assert_matches_oracle(y, ref, what="op eager")
    torch.testing.assert_close(y, kl.quant_linear(x, p), rtol=0, atol=0)
    # captured in a CUDA graph (output buffer fixed by linear_out)
    out = torch.empty_like(y)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        torch.ops.kl_b200.linear_out(x, p.data, p.scales, None, None, N.KL_W8_ROW, k, False, False, N.KL_FLAG_PDL, out)
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, y, rtol=0, atol=0)
    # traced by torch.compile (the op is opaque to the compiler; no Triton codegen)
    fn = torch.compile(lambda a: kl.quant_linear(a, p) * 2, backend="aot_eager", fullgraph=True)
    torch.testing.assert_close(fn(x), y * 2, rtol=0, atol=0)


@pytest.mark.gpu
def test_reference_ops_through_dispatcher():
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1024, generator=gen).bfloat16().cuda()
    w = (torch.randn(256, 1024, generator=gen) * 0.02).bfloat16().cuda()
    y = torch.ops.kl_b200.project(x, w, None, None, 128, 4, False, False)
    torch.testing.assert_close(y, kl.project(x, w), rtol=0, atol=0)
    pk = kl.quantize_int4((torch.randn(512, 1024, generator=gen) * 0.02).cuda(), 128)
    torch.testing.assert_close(torch.ops.kl_b200.int4_gemv(x, pk.data, pk.scales, 128, 32), kl.int4_gemv(x, pk),
                               rtol=0, atol=0)
    v, i = torch.ops.kl_b200.int4_lm_head_topk(x, pk.data, pk.scales, 128, 4, 32)
    v2, i2 = kl.int4_lm_head_topk(x, pk, 4)
    torch.testing.assert_close(v, v2, rtol=0, atol=0)
    assert torch.equal(i, i2)


@pytest.mark.gpu
def test_streams_get_their_own_workspace():
    """Persistent-kernel calls on two streams use different scratch buffers."""
    gen = torch.Generator().manual_seed(2)
    p = kl.quantize_int8_rowwise((torch.randn(151936, 1024, generator=gen) * 0.02).cuda())
    x = torch.randn(4, 1024, generator=gen).bfloat16().cuda()
    ref = kl.quant_linear(x, p)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    for s in (s1, s2):
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            outs.append(kl.quant_linear(x, p))
    torch.cuda.synchronize()
    for o in outs:
        torch.testing.assert_close(o, ref, rtol=0, atol=0)
    keys = [k for k in N._workspaces if isinstance(k, tuple)]
    assert {k[1] for k in keys} >= {s1.cuda_stream, s2.cuda_stream}
