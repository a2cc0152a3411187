"""Head-parallel Gemma-4 attention: one process per GPU, each owning a share of
the query heads together with their KV heads.

The attention path has no exchange step while every rank owns whole KV heads
(local layers 32Q/16KV up to 16 ranks; global layers 32Q/4KV up to 4 ranks):
forward and backward run on the local shard only.  When there are more ranks
than KV heads (global layers on 8 GPUs), the ranks of one KV group share that
KV head and each computes the dK/dV contribution of its own query heads; the
one exchange is the sum of those partial dK/dV over the sharing ranks
(``reduce_kv_grads``), an all-reduce inside a process subgroup of 2 ranks.
The forward and dQ never communicate.

The per-rank compute is ``ops.attn_fwd`` / ``ops.attn_bwd`` (the CUDA kernels);
callers may pass other callables with the same signature, which is how the
sharding and reduction logic is tested on CPU with ``gloo``.

Reference behaviour kept: the head-to-KV-group assignment of grouped-query
attention (query head h reads KV head h // (Hq / Hkv), reference.py:38-61
expands K/V the same way).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch


@dataclass(frozen=True)
class HeadShard:
    """One rank's heads: query heads [q_start, q_stop) and KV heads
    [kv_start, kv_stop); ``kv_peers`` lists the ranks holding the same KV heads
    (just this rank when it owns them alone)."""

    world_size: int
    rank: int
    q_start: int
    q_stop: int
    kv_start: int
    kv_stop: int
    kv_peers: tuple[int, ...]

    @property
    def num_q_heads(self) -> int:
        return self.q_stop - self.q_start

    @property
    def num_kv_heads(self) -> int:
        return self.kv_stop - self.kv_start

    @property
    def shares_kv(self) -> bool:
        return len(self.kv_peers) > 1


def head_shard(num_q_heads: int, num_kv_heads: int, world_size: int, rank: int) -> HeadShard:
    """Split query heads evenly over ``world_size`` ranks, keeping every query
    head with its KV head (GQA group = num_q_heads / num_kv_heads)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank out of range")
    if num_kv_heads <= 0 or num_q_heads % num_kv_heads:
        raise ValueError("query heads must be a positive multiple of KV heads")
    if num_q_heads % world_size:
        raise ValueError("query heads must divide evenly over the ranks")
    group = num_q_heads // num_kv_heads
    q_per = num_q_heads // world_size
    q_start = rank * q_per
    if q_per >= group:
        if q_per % group:
            raise ValueError("a rank's query heads must cover whole KV groups")
        kv_per = q_per // group
        kv_start = rank * kv_per
        return HeadShard(world_size, rank, q_start, q_start + q_per, kv_start, kv_start + kv_per,
                         (rank,))
    if group % q_per:
        raise ValueError("ranks sharing a KV head must split its query group evenly")
    ranks_per_kv = group // q_per
    kv = q_start // group
    first = kv * ranks_per_kv
    return HeadShard(world_size, rank, q_start, q_start + q_per, kv, kv + 1,
                     tuple(range(first, first + ranks_per_kv)))


class HeadParallelGroup:
    """Process subgroups for the dK/dV reduction of one head-parallel layer.

    Construction is collective: every rank of ``group`` must build the same
    layers in the same order (``torch.distributed.new_group`` is called for
    every set of KV-sharing ranks on every rank)."""

    def __init__(self, num_q_heads: int, num_kv_heads: int, group=None):
        import torch.distributed as dist

        self._dist = dist
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.shard = head_shard(num_q_heads, num_kv_heads, world, rank)
        peer_sets = sorted({head_shard(num_q_heads, num_kv_heads, world, r).kv_peers
                            for r in range(world)})
        self.kv_group = None
        for peers in peer_sets:
            if len(peers) > 1:
                global_ranks = [dist.get_global_rank(group, r) if group is not None else r
                                for r in peers]
                pg = dist.new_group(ranks=global_ranks)
                if rank in peers:
                    self.kv_group = pg

    def local_heads(self, x: torch.Tensor, kind: str, head_dim: int = 2) -> torch.Tensor:
        """This rank's query (kind="q") or KV (kind="kv") heads of a full tensor."""
        s = self.shard
        lo, hi = (s.q_start, s.q_stop) if kind == "q" else (s.kv_start, s.kv_stop)
        return x.narrow(head_dim, lo, hi - lo)

    def reduce_kv_grads(self, dk: torch.Tensor, dv: torch.Tensor) -> None:
        """Sum the partial dK/dV of the ranks sharing this rank's KV heads (in place)."""
        if self.kv_group is None:
            return
        self._dist.all_reduce(dk, group=self.kv_group)
        self._dist.all_reduce(dv, group=self.kv_group)


def head_parallel_forward(hp: HeadParallelGroup, q, k, v, *, window: int,
                          attn_fwd: Callable | None = None):
    """Forward of the local shard (q: this rank's query heads, k/v: its KV heads)."""
    if attn_fwd is None:
        from . import ops

        attn_fwd = ops.attn_fwd
    return attn_fwd(q, k, v, window=window)


def head_parallel_backward(hp: HeadParallelGroup, q, k, v, out, lse, dout, *, window: int,
                           attn_bwd: Callable | None = None):
    """Backward of the local shard; dK/dV are complete (summed over the ranks
    sharing the KV heads) on return."""
    if attn_bwd is None:
        from . import ops

        attn_bwd = ops.attn_bwd
    dq, dk, dv = attn_bwd(q, k, v, out, lse, dout, window=window)
    hp.reduce_kv_grads(dk, dv)
    return dq, dk, dv
