"""The fused lm_head top-k (``lm_head_topk`` / ``kl_linear_topk``): the tcgen05
GEMM's epilogue selects each 128-row tile's candidates and the logits are
never written (the reference's ``_head_candidates`` +
``int4_lm_head_topk``, ``learning/09_int4/kernels.py:37-50,77-99``).

Exactness: values and ids equal the top-k, lowest index first on ties, of the
logits the same kernel writes when asked for them (``quant_linear``), and
agree with the fp32 oracle wherever its decision is clear."""
import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import load_kl

kl = load_kl()
N = kl._native
pytestmark = pytest.mark.gpu


def _weights(n, k, fmt, seed):
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=gen) * 0.02
    if n > 40:                                   # exact ties between distant rows
        w[n // 2 + 3] = w[5]
        w[n - 1] = w[n // 3]
    p = kl.quantize_int4_asym(w.cuda(), 128) if fmt == "w4_asym" else kl.quantize_int8_rowwise(w.cuda())
    return p, gen


def _expected(logits, k):
    out_v, out_i = [], []
    for row in logits:
        v, i = O.topk_lowest_index(row, k)
        out_v.append(v)
        out_i.append(i)
    return np.stack(out_v), np.stack(out_i)


@pytest.mark.parametrize("fmt,n,kdim,m,topk", [
    ("w8_row", 151936, 1024, 1, 1), ("w8_row", 151936, 1024, 1, 8), ("w8_row", 151936, 1024, 8, 4),
    ("w8_row", 151936, 1024, 64, 8), ("w8_row", 128256, 3072, 2, 8), ("w8_row", 30000, 1024, 200, 2),
    ("w4_asym", 151936, 1024, 1, 8), ("w4_asym", 151936, 1024, 16, 4),
    ("w8_row", 1000, 256, 3, 8), ("w8_row", 5, 128, 2, 5),
])
def test_matches_topk_of_the_logits(fmt, n, kdim, m, topk):
    p, gen = _weights(n, kdim, fmt, seed=n + m)
    x = torch.randn(m, kdim, generator=gen).bfloat16().cuda()
    v, i = kl.lm_head_topk(x, p, topk)
    # the logits from the same kernel and plan (the persistent tcgen05 GEMM)
    logits = kl.quant_linear(x, p, path="persistent" if fmt == "w8_row" else None).float().cpu().numpy()
    ev, ei = _expected(logits, topk)
    np.testing.assert_array_equal(i.cpu().numpy(), ei)
    np.testing.assert_array_equal(v.cpu().numpy(), ev)
    # against the fp32 oracle: same ids wherever the k-th / (k+1)-th margin is clear
    if fmt == "w8_row" and n * kdim <= 151936 * 1024:
        deq = O.dequantize_int8_rowwise(p.data.cpu().numpy(), p.scales.float().cpu().numpy())
        ref = O.linear_f32(x.float().cpu().numpy(), deq)
        srt = -np.sort(-ref, axis=1)
        for r in range(m):
            if topk < n and srt[r, topk - 1] - srt[r, topk] > 0.05:
                assert set(i[r].cpu().numpy()) == set(np.argsort(-ref[r], kind="stable")[:topk])
    assert N.device_status(0) == 0


def test_packed_candidates_and_offset():
    p, gen = _weights(75968, 1024, "w8_row", seed=7)
    x = torch.randn(4, 1024, generator=gen).bfloat16().cuda()
    v, i = kl.lm_head_topk(x, p, 8, index_offset=75968)
    packed = kl.lm_head_topk(x, p, 8, index_offset=75968, packed=True)
    assert packed.dtype == torch.int64 and packed.shape == (4, 8)
    ids = (packed >> 32).cpu()
    vals = (packed & 0xFFFFFFFF).to(torch.int32).view(torch.float32).cpu()
    assert torch.equal(ids, i.cpu())
    assert torch.equal(vals, v.cpu())
    assert int(i.min()) >= 75968
    # merging one rank's packed candidates gives the same top-k back
    mv, mi = kl.sharded_head.topk_merge_rows(packed, 8)
    assert torch.equal(mi, i) and torch.equal(mv, v)


def test_sharded_head_uses_the_fused_selection():
    gen = torch.Generator().manual_seed(21)
    w = (torch.randn(151936, 1024, generator=gen) * 0.02).cuda()
    x = torch.randn(8, 1024, generator=gen).bfloat16().cuda()
    head = kl.VocabShardedHead.from_full_weight(w)
    v, i = head.topk(x, 8)
    fv, fi = kl.lm_head_topk(x, head.weight, 8)
    assert torch.equal(i, fi) and torch.equal(v, fv)


def test_rejects_what_it_does_not_take():
    p, gen = _weights(1000, 256, "w8_row", seed=1)
    with pytest.raises(ValueError):
        kl.lm_head_topk(torch.randn(1, 256).bfloat16().cuda(), p, 9)
    with pytest.raises(RuntimeError):
        kl.lm_head_topk(torch.randn(1, 256).half().cuda(), p, 1)     # bf16 activations only
