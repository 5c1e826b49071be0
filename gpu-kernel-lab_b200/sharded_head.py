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

from .linear import QuantLinear, quant_linear


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

    def __init__(self, weight_shard, vocab: int, *, group=None, fmt: str = "w8_row", project=None):
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

    @classmethod
    def from_full_weight(cls, weight: torch.Tensor, *, group=None, fmt: str = "w8_row", project=None):
        """Cut this rank's rows out of the full ``[V, K]`` matrix and quantize them."""
        import torch.distributed as dist
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        lo, hi = shard_bounds(weight.shape[0], world, rank)
        return cls(weight[lo:hi].contiguous(), weight.shape[0], group=group, fmt=fmt, project=project)

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
