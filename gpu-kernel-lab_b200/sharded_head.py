"""Vocab-sharded quantized lm_head with an NCCL all-gather of the logits.

The lm_head ``W[V, K]`` is split by rows (vocabulary entries, i.e. columns of
the logits) over the ranks of a process group: rank ``r`` holds rows
``[r*V/G, (r+1)*V/G)``, quantized.  Each rank computes its shard of the logits
in the kernel's transposed layout ``[V/G, M]`` (swap-AB writes it contiguously),
and ``all_gather_into_tensor`` concatenates the shards into ``[V, M]`` in rank
order, which IS the full transposed logits; the result is returned as the
``[M, V]`` view.  No shard is reshaped or copied before the collective.

V must divide evenly by the world size (151,936 over 2/4/8 and 128,256 over
2/4/8 do).  The local projection defaults to this package's kernels; tests on
CPU pass their own ``project`` callable.
"""
from __future__ import annotations

import torch

from . import _native as N
from .linear import QuantLinear, lm_head_topk, quant_linear


def topk_rows(logits: torch.Tensor, k: int, index_offset: int = 0, *, packed: bool = False):
    """Per-row top-k of ``logits [rows, n]`` (bf16/f16) on the GPU: values (f32)
    descending, the lower index first on ties; ids are column + ``index_offset``.
    Returns ``(values, ids)``, or with ``packed`` one int64 ``[rows, k]`` tensor of
    ``id << 32 | value bits`` pairs (the form :func:`topk_merge_rows` takes)."""
    if logits.ndim != 2 or not logits.is_cuda or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous CUDA [rows, n] tensor")
    rows, n = logits.shape
    lib = N.lib()
    ws = torch.empty(max(1, lib.kl_topk_rows_workspace_bytes(rows, n, k)), dtype=torch.uint8, device=logits.device)
    values = None if packed else torch.empty(rows, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(rows, k, dtype=torch.int64, device=logits.device)
    N.check(lib.kl_topk_rows(N.ptr(logits), N.act_dtype_code(logits.dtype), rows, n, n, index_offset, k,
                             N.ptr(values), N.ptr(ids), N.ptr(ws), ws.numel(), N.stream_handle(logits.device)))
    return ids if packed else (values, ids)


def topk_merge_rows(packed: torch.Tensor, k: int):
    """Global top-k of each row of packed candidates (int64 ``[rows, count]``)."""
    if packed.ndim != 2 or packed.dtype != torch.int64 or not packed.is_cuda:
        raise ValueError("packed candidates must be a CUDA int64 [rows, count] tensor")
    packed = packed.contiguous()
    rows, count = packed.shape
    out_v = torch.empty(rows, k, dtype=torch.float32, device=packed.device)
    out_i = torch.empty(rows, k, dtype=torch.int64, device=packed.device)
    N.check(N.lib().kl_topk_merge_rows(N.ptr(packed), rows, count, k, N.ptr(out_v), N.ptr(out_i),
                                       N.stream_handle(packed.device)))
    return out_v, out_i


def _fused_local_topk(x, w, k, offset):
    """This shard's top-k per token, packed, from the fused lm_head top-k (no
    logits written); shapes or formats the tcgen05 kernel does not take
    compute the shard's logits and select from them."""
    try:
        return lm_head_topk(x, w, k, index_offset=offset, packed=True)
    except N.NativeError as e:
        if e.status != N.KL_ERR_UNSUPPORTED:
            raise
    return topk_rows(quant_linear(x, w), k, offset, packed=True)


def shard_bounds(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Row range ``[lo, hi)`` of ``rank``'s shard; requires an even split."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if vocab % world:
        raise ValueError(f"vocabulary {vocab} does not split evenly over {world} ranks")
    per = vocab // world
    return rank * per, (rank + 1) * per


class VocabShardedHead:
    """One rank's shard of a quantized lm_head plus the gather.

    ``weight_shard``: this rank's rows, already quantized (any format
    ``quant_linear`` takes) or a dense tensor together with ``fmt``.
    """

    def __init__(self, weight_shard, vocab: int, *, group=None, fmt: str = "w8_row", project=None,
                 local_topk=None, merge_topk=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        lo, hi = shard_bounds(vocab, self.world, self.rank)
        self.vocab, self.lo, self.hi = vocab, lo, hi
        if isinstance(weight_shard, torch.Tensor):
            if weight_shard.shape[0] != hi - lo:
                raise ValueError(f"shard has {weight_shard.shape[0]} rows, expected {hi - lo}")
            weight_shard = QuantLinear.from_weight(weight_shard, fmt).weight_q
        self.weight = weight_shard
        self.project = project or (lambda x, w, out: quant_linear(x, w, transposed=True, out=out))
        # local_topk(x, w, k, offset) -> packed int64 [M, k]; merge_topk(packed [M, G*k], k) -> (values, ids)
        self.local_topk = local_topk or _fused_local_topk
        self.merge_topk = merge_topk or topk_merge_rows

    @classmethod
    def from_full_weight(cls, weight: torch.Tensor, *, group=None, fmt: str = "w8_row", **hooks):
        """Cut this rank's rows out of the full ``[V, K]`` matrix and quantize them."""
        import torch.distributed as dist
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        lo, hi = shard_bounds(weight.shape[0], world, rank)
        return cls(weight[lo:hi].contiguous(), weight.shape[0], group=group, fmt=fmt, **hooks)

    def topk(self, x: torch.Tensor, k: int = 1):
        """Global top-k of the logits without gathering them: every rank takes the
        top-k of its shard (ids offset by its first row), the ranks all-gather
        those ``M x k`` candidates (``G·M·k·8`` bytes instead of ``M·V·2``), and
        every rank merges them.  Values f32 ``[M, k]``, ids int64 ``[M, k]``;
        ties go to the lower vocabulary index."""
        x2 = x.reshape(-1, x.shape[-1])
        m = x2.shape[0]
        packed = self.local_topk(x2, self.weight, k, self.lo)       # [M, k] int64: id << 32 | value bits
        if self.world > 1:
            # gathered in rank order along the first dimension: [world * M, k]
            gp = torch.empty(self.world * m, k, dtype=torch.int64, device=packed.device)
            self.dist.all_gather_into_tensor(gp, packed.contiguous(), group=self.group)
            packed = gp.view(self.world, m, k).permute(1, 0, 2).reshape(m, self.world * k)
        return self.merge_topk(packed.contiguous(), k)

    def local_logits(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's shard, transposed: ``[V/G, M]``."""
        x2 = x.reshape(-1, x.shape[-1])
        if out is None:
            out = torch.empty(self.hi - self.lo, x2.shape[0], dtype=x.dtype, device=x.device)
        return self.project(x2, self.weight, out)

    def __call__(self, x: torch.Tensor, *, gathered: torch.Tensor | None = None) -> torch.Tensor:
        """Full logits ``[..., V]`` (a transposed view of the gathered ``[V, M]``)."""
        lead = x.shape[:-1]
        shard = self.local_logits(x)
        m = shard.shape[1]
        if gathered is None:
            gathered = torch.empty(self.vocab, m, dtype=shard.dtype, device=shard.device)
        if self.world == 1:
            gathered.copy_(shard)
        else:
            self.dist.all_gather_into_tensor(gathered, shard, group=self.group)
        return gathered.t().reshape(*lead, self.vocab) if len(lead) != 1 else gathered.t()
