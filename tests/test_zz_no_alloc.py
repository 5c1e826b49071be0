"""kl_linear_noalloc, the int8 row-scale linear for callers that cannot allocate
device memory: an FFI binding that only receives the model's tensors from a host
runtime owning all device allocation, or code running while another library
captures a CUDA graph.  It keeps its scratch in a device array inside the
library instead of a caller-supplied workspace.

Each check calls both entry points through the C ABI: the new one against
kl_linear with a caller-owned workspace, on several calls in a row (the static
scratch keeps the previous call's contents).  The file name puts it last in
collection; it passes alone in a fresh process too.
"""
import ctypes

import pytest
import torch

from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
N = kl._native
pytestmark = pytest.mark.gpu


def _weights(n, k, seed):
    gen = torch.Generator().manual_seed(seed)
    return kl.quantize_int8_rowwise((torch.randn(n, k, generator=gen) * 0.02).cuda())


def _noalloc(x, p, swiglu, y):
    lib = N.lib()
    m, k = x.shape
    return lib.kl_linear_noalloc(N.ptr(x), N.act_dtype_code(x.dtype), m, k, N.ptr(p.data), p.data.shape[0],
                                 N.ptr(p.scales), int(swiglu), N.ptr(y), N.stream_handle(x.device))


def _with_workspace(x, p, swiglu):
    """The existing entry point, given a workspace this test allocates."""
    lib = N.lib()
    m, k = x.shape
    n = p.data.shape[0]
    y = torch.empty(m, n // 2 if swiglu else n, device=x.device, dtype=x.dtype)
    nbytes = lib.kl_linear_workspace_bytes(m, n, k, N.KL_W8_ROW, int(swiglu), 0)
    ws = torch.zeros(max(nbytes, 1), device=x.device, dtype=torch.uint8)
    N.check(lib.kl_linear(N.ptr(x), N.act_dtype_code(x.dtype), m, k, N.ptr(p.data), N.KL_W8_ROW, n, k,
                          N.ptr(p.scales), None, None, int(swiglu), N.ptr(y), N.ptr(ws), ctypes.c_size_t(nbytes), 0,
                          N.stream_handle(x.device)))
    return y


# (m, n, k, swiglu): split tiles at M = 1 (stream-K partials in the scratch), a
# SwiGLU gate/up at a ragged M, the widest N at the largest accepted M.
CASES = [(1, 4096, 1024, False), (37, 6144, 1024, True), (64, 151936, 1024, False), (8, 1024, 3072, False)]


def test_noalloc_matches_kl_linear_on_consecutive_calls():
    torch.manual_seed(0)
    probs = []
    for i, (m, n, k, sw) in enumerate(CASES):
        p = _weights(n, k, seed=100 + i)
        x = torch.randn(m, k, device="cuda").bfloat16()
        ref = _with_workspace(x, p, sw)
        probs.append((x, p, sw, ref))
    torch.cuda.synchronize()
    # every case twice in a row, then the whole list again in reverse order
    order = [0, 0, 1, 1, 2, 2, 3, 3, 3, 2, 1, 0]
    for idx in order:
        x, p, sw, ref = probs[idx]
        y = torch.full_like(ref, float("nan"))
        N.check(_noalloc(x, p, sw, y))
        torch.cuda.synchronize()
        assert_matches_oracle(y, ref.float().cpu().numpy(), what=f"noalloc case {idx} {CASES[idx]}")
    assert N.device_status(0, reset=False) == 0


def test_noalloc_f16_activations():
    p = _weights(2048, 1024, seed=7)
    x = torch.randn(16, 1024, device="cuda").half()
    ref = _with_workspace(x, p, False)
    for _ in range(2):
        y = torch.empty_like(ref)
        N.check(_noalloc(x, p, False, y))
        torch.cuda.synchronize()
        assert_matches_oracle(y, ref.float().cpu().numpy(), what="noalloc f16")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    p = _weights(256, 256, seed=8)
    x = torch.randn(65, 256, device="cuda").bfloat16()
    y = torch.empty(65, 256, device="cuda", dtype=torch.bfloat16)
    assert _noalloc(x, p, False, y) == N.KL_ERR_INVALID
    assert b"m <= 64" in N.lib().kl_last_error()
