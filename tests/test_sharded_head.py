"""Vocab-sharded lm_head: shard bounds, gather order and equality with the
unsharded head, as world-size-2 ``gloo`` ranks on CPU (the local projection is
the dequantise-then-matmul reference, supplied by the test)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import quant_oracle as O
from tests.conftest import load_kl

kl = load_kl()


def test_shard_bounds():
    sb = kl.sharded_head.shard_bounds
    assert sb(151936, 8, 0) == (0, 18992) and sb(151936, 8, 7) == (132944, 151936)
    assert sb(128256, 4, 2) == (64128, 96192)
    with pytest.raises(ValueError, match="evenly"):
        sb(1001, 2, 0)
    with pytest.raises(ValueError):
        sb(1000, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_project(x, w, out):
    deq = kl.dequantize_int8_rowwise(w).float()
    out.copy_((x.float() @ deq.t()).t().to(out.dtype))
    return out


def _rank_main(rank, world, port, vocab, k, m_list, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(7)
        w = torch.randn(vocab, k, generator=gen) * 0.02             # same full matrix on every rank
        head = kl.VocabShardedHead.from_full_weight(w, project=_cpu_project)
        assert (head.lo, head.hi) == kl.sharded_head.shard_bounds(vocab, world, rank)
        out = {}
        for m in m_list:
            x = torch.randn(m, k, generator=torch.Generator().manual_seed(100 + m)).to(torch.float32)
            out[m] = head(x).clone()
            # the ranks agree on the gathered logits
            ref = out[m].clone()
            dist.broadcast(ref, src=0)
            assert torch.equal(ref, out[m])
        results[rank] = {m: v.numpy() for m, v in out.items()}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gathered_logits_equal_unsharded(world):
    vocab, k, m_list = 512, 64, [1, 5]
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, vocab, k, m_list, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        got = dict(results)
    w = torch.randn(vocab, k, generator=torch.Generator().manual_seed(7)) * 0.02
    full = kl.quantize_int8_rowwise(w)
    for m in m_list:
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(100 + m))
        ref = (x @ kl.dequantize_int8_rowwise(full).float().t()).numpy()
        for r in range(world):
            np.testing.assert_allclose(got[r][m], ref, rtol=1e-5, atol=1e-6)
            assert (got[r][m].argmax(-1) == ref.argmax(-1)).all()




@pytest.mark.gpu
@pytest.mark.parametrize("m", [1, 16, 64])
def test_single_gpu_head_matches_quant_linear(m):
    """World size 1: the transposed shard path gives the plain kernel's logits."""
    gen = torch.Generator().manual_seed(m)
    w = (torch.randn(151936, 1024, generator=gen) * 0.02).cuda()
    x = torch.randn(m, 1024, generator=gen).bfloat16().cuda()
    head = kl.VocabShardedHead.from_full_weight(w)
    got = head(x)
    ref = kl.quant_linear(x, head.weight)
    assert got.shape == (m, 151936)
    torch.testing.assert_close(got, ref, rtol=0, atol=0)


def _nccl_rank(rank, world, port, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator().manual_seed(11)
        w = (torch.randn(128256, 3072, generator=gen) * 0.02).cuda()
        x = torch.randn(8, 3072, generator=gen).bfloat16().cuda()
        head = kl.VocabShardedHead.from_full_weight(w)
        logits = head(x)
        full = kl.quant_linear(x, kl.quantize_int8_rowwise(w))
        torch.cuda.synchronize()
        # split tiles may sum their partials in a different grouping than the
        # unsharded launch: compare within the north-star tolerance
        close = (logits.float() - full.float()).abs().max().item() <= 2e-2
        v, i = head.topk(x, 4)
        fv, fi = kl.sharded_head.topk_rows(logits.contiguous(), 4)   # top-k of the gathered logits
        same = bool(torch.equal(i, fi)) and bool(torch.equal(v, fv))
        results[rank] = (close and same, bool((logits.argmax(-1) == full.argmax(-1)).all()))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_nccl_gather_equals_single_gpu_head():
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert all(results[r] == (True, True) for r in range(2)), dict(results)


# ---------------------------------------------------------------- sharded top-k
def _pack(v, i):
    return (torch.as_tensor(i, dtype=torch.int64) << 32) | (
        torch.as_tensor(v, dtype=torch.float32).view(torch.int32).to(torch.int64) & 0xFFFFFFFF)


def _unpack(p):
    low = p & 0xFFFFFFFF
    return torch.where(low >= 2 ** 31, low - 2 ** 32, low).to(torch.int32).view(torch.float32), p >> 32


def _cpu_local_topk(x, w, k, offset):
    """Shard top-k on the CPU, packed like the kernel's output."""
    logits = (x.float() @ kl.dequantize_int8_rowwise(w).float().t())
    logits = logits.to(torch.bfloat16).float()                   # the kernel's output rounding
    vals, ids = [], []
    for row in logits.numpy():
        v, i = O.topk_lowest_index(row, k)
        vals.append(v); ids.append(i + offset)
    return _pack(np.array(vals), np.array(ids))


def _cpu_merge_topk(packed, k):
    cv, ci = _unpack(packed)
    vals, ids = [], []
    for v, i in zip(cv.numpy(), ci.numpy()):
        order = np.lexsort((i, -v))[:k]                          # value descending, then lower index
        vals.append(v[order]); ids.append(i[order])
    return torch.tensor(np.array(vals)), torch.tensor(np.array(ids))


def _rank_topk(rank, world, port, vocab, k, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(3)
        w = torch.randn(vocab, 64, generator=gen) * 0.02
        w[vocab // 2 + 5] = w[7]                                 # the same row in both shards: a cross-shard tie
        head = kl.VocabShardedHead.from_full_weight(w, local_topk=_cpu_local_topk, merge_topk=_cpu_merge_topk)
        x = torch.randn(4, 64, generator=torch.Generator().manual_seed(4))
        v, i = head.topk(x, k)
        results[rank] = (v.numpy(), i.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_topk_equals_full_topk():
    vocab, k, world = 512, 4, 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_rank_topk, args=(r, world, port, vocab, k, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        got = dict(results)
    gen = torch.Generator().manual_seed(3)
    w = torch.randn(vocab, 64, generator=gen) * 0.02
    w[vocab // 2 + 5] = w[7]
    x = torch.randn(4, 64, generator=torch.Generator().manual_seed(4))
    full = kl.quantize_int8_rowwise(w)
    ref_v, ref_i = _unpack(_cpu_local_topk(x, full, k, 0))
    for r in range(world):
        np.testing.assert_array_equal(got[r][1], ref_i.numpy())
        np.testing.assert_array_equal(got[r][0], ref_v.numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n,k,offset", [(1, 151936, 1, 0), (8, 75968, 4, 75968), (3, 1000, 8, 5)])
def test_topk_rows_kernel(rows, n, k, offset):
    gen = torch.Generator().manual_seed(rows + n)
    logits = torch.randn(rows, n, generator=gen).bfloat16()
    logits[:, n // 3] = logits.max() + 1                         # a tie between two columns
    logits[:, n // 2] = logits[:, n // 3]
    v, i = kl.sharded_head.topk_rows(logits.cuda(), k, offset)
    for r in range(rows):
        rv, ri = O.topk_lowest_index(logits[r].float().numpy(), k)
        np.testing.assert_array_equal(i[r].cpu().numpy(), ri + offset)
        np.testing.assert_array_equal(v[r].cpu().numpy(), rv)


@pytest.mark.gpu
def test_single_gpu_head_topk():
    gen = torch.Generator().manual_seed(21)
    w = (torch.randn(151936, 1024, generator=gen) * 0.02).cuda()
    x = torch.randn(8, 1024, generator=gen).bfloat16().cuda()
    head = kl.VocabShardedHead.from_full_weight(w)
    v, i = head.topk(x, 4)
    logits = head(x).float().cpu().numpy()
    for r in range(8):
        rv, ri = O.topk_lowest_index(logits[r], 4)
        np.testing.assert_array_equal(i[r].cpu().numpy(), ri)
