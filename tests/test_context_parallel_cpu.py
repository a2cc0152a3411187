"""Context parallelism on CPU ranks (``gloo``): the ring schedule of global
layers and the halo exchange of sliding-window layers, with float64 CPU block
computations standing in for the kernels (``cp_cpu_blocks.CpuBlocks``).

Every rank checks its shard of the output, LSE and gradients against the
whole-sequence float64 oracle.  World sizes 2 and 3 cover every kind of ring
step (diagonal blocks, key chunks before both query chunks, key chunks between
them) and the dK/dV accumulators' full trip round the ring."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from gemma4_fa4_kernels_b200.context_parallel import zigzag_shard, zigzag_unshard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_zigzag_shards_round_trip():
    x = torch.arange(2 * 3 * 5).reshape(1, 30, 1, 1)
    parts = [zigzag_shard(x, r, 3) for r in range(3)]
    assert parts[0][0, :, 0, 0].tolist() == [0, 1, 2, 3, 4, 25, 26, 27, 28, 29]
    assert torch.equal(zigzag_unshard(parts), x)
    with pytest.raises(ValueError):
        zigzag_shard(x, 0, 4)


def _inputs(s, hq, hkv, d, seed=3):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, s, hq, d, generator=g, dtype=torch.float64)
    k = torch.randn(1, s, hkv, d, generator=g, dtype=torch.float64)
    v = torch.randn(1, s, hkv, d, generator=g, dtype=torch.float64)
    do = torch.randn(1, s, hq, d, generator=g, dtype=torch.float64)
    dlse = torch.randn(1, hq, s, generator=g, dtype=torch.float64)
    return q, k, v, do, dlse


def _close(a, b, tol=2e-6):
    # the running output, LSE and gradient accumulators are fp32 (as on the GPU)
    np.testing.assert_allclose(a.double().numpy(), b.double().numpy(), rtol=tol, atol=tol)


def _ring_main(rank, world, port, use_dlse):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cp_cpu_blocks import CpuBlocks, reference

        from gemma4_fa4_kernels_b200.context_parallel import (ring_global_backward,
                                                              ring_global_forward)

        s, hq, hkv, d = 2 * world * 7, 4, 2, 8
        q, k, v, do, dlse = _inputs(s, hq, hkv, d)
        dlse = dlse if use_dlse else None
        ro, rl, rq, rk, rv = reference(q, k, v, do, dlse=dlse)
        sh = lambda x: zigzag_shard(x, rank, world)  # noqa: E731
        shl = lambda x: zigzag_shard(x, rank, world, dim=2)  # noqa: E731
        blocks = CpuBlocks()
        o, lse = ring_global_forward(sh(q), sh(k), sh(v), blocks=blocks)
        _close(o, sh(ro))
        _close(lse, shl(rl), tol=2e-5)
        # the backward takes the exact final O / LSE (the CPU blocks keep float64)
        dq, dk, dv = ring_global_backward(sh(q), sh(k), sh(v), sh(ro), shl(rl), sh(do),
                                          None if dlse is None else shl(dlse), blocks=blocks)
        _close(dq, sh(rq), tol=2e-6)
        _close(dk, sh(rk), tol=2e-6)
        _close(dv, sh(rv), tol=2e-6)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,use_dlse", [(2, False), (3, True)], ids=["two", "three_dlse"])
def test_ring_global_attention_matches_the_oracle(world, use_dlse):
    mp.spawn(_ring_main, args=(world, _free_port(), use_dlse), nprocs=world, join=True)


def _halo_main(rank, world, port, meta):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cp_cpu_blocks import CpuBlocks, reference

        from gemma4_fa4_kernels_b200.context_parallel import (halo_local_backward,
                                                              halo_local_forward)

        window, c, hq, hkv, d = 6, 9, 4, 2, 8
        s = world * c
        q, k, v, do, _ = _inputs(s, hq, hkv, d, seed=5)
        vis = doc = None
        if meta:
            vis = torch.full((s,), -1, dtype=torch.int32)
            vis[2:6] = 0          # images inside rank 0's chunk
            vis[c + 3:c + 8] = 1  # and inside rank 1's
            doc = torch.zeros(s, dtype=torch.int32)
            doc[c + 5:] = 1       # a document boundary inside rank 1's chunk
        ro, rl, rq, rk, rv = reference(q, k, v, do, window=window, vision_ids=vis,
                                       document_ids=doc)
        rows = slice(rank * c, (rank + 1) * c)
        blocks = CpuBlocks()
        o, lse = halo_local_forward(q[:, rows], k[:, rows], v[:, rows], window=window,
                                    vision_ids=vis, document_ids=doc, blocks=blocks)
        _close(o, ro[:, rows])
        _close(lse, rl[:, :, rows], tol=2e-5)
        dq, dk, dv = halo_local_backward(q[:, rows], k[:, rows], v[:, rows], ro[:, rows],
                                         rl[:, :, rows], do[:, rows], window=window,
                                         vision_ids=vis, document_ids=doc, blocks=blocks)
        _close(dq, rq[:, rows], tol=2e-6)
        _close(dk, rk[:, rows], tol=2e-6)
        _close(dv, rv[:, rows], tol=2e-6)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,meta", [(2, False), (3, True)], ids=["text", "vision_docs"])
def test_halo_local_attention_matches_the_oracle(world, meta):
    mp.spawn(_halo_main, args=(world, _free_port(), meta), nprocs=world, join=True)


def _cross_main(rank, world, port):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cp_cpu_blocks import CpuBlocks

        from gemma4_fa4_kernels_b200.context_parallel import halo_local_forward
        from gemma4_fa4_kernels_b200.errors import UnsupportedB200Path

        c = 9
        q, k, v, _, _ = _inputs(2 * c, 2, 1, 8)
        vis = torch.full((2 * c,), -1, dtype=torch.int32)
        vis[c - 2:c + 2] = 4  # one image across the shard boundary
        rows = slice(rank * c, (rank + 1) * c)
        with pytest.raises(UnsupportedB200Path):
            halo_local_forward(q[:, rows], k[:, rows], v[:, rows], window=6, vision_ids=vis,
                               blocks=CpuBlocks())
    finally:
        dist.destroy_process_group()


def test_halo_rejects_an_image_across_shards_before_any_exchange():
    mp.spawn(_cross_main, args=(2, _free_port()), nprocs=2, join=True)
