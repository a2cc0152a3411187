"""Head-parallel sharding and the dK/dV exchange on CPU: world_size-2 ``gloo``
ranks, the oracle standing in for the per-rank CUDA compute, checked against
the full single-process oracle result.  Also covers the multi-rank plumbing
that bench.py uses (barrier, max over ranks)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from gemma4_fa4_kernels_b200.head_parallel import head_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------- shard arithmetic
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_local_layer_shards_own_whole_kv_heads(world):
    shards = [head_shard(32, 16, world, r) for r in range(world)]
    assert [s.q_start for s in shards] == [r * 32 // world for r in range(world)]
    assert all(not s.shares_kv for s in shards)
    covered = sorted(h for s in shards for h in range(s.kv_start, s.kv_stop))
    assert covered == list(range(16))
    for s in shards:  # every query head stays with its KV head (group 2)
        assert all(s.kv_start <= h // 2 < s.kv_stop for h in range(s.q_start, s.q_stop))


def test_global_layer_on_eight_ranks_shares_kv_in_pairs():
    shards = [head_shard(32, 4, 8, r) for r in range(8)]
    assert [s.kv_peers for s in shards] == [(0, 1), (0, 1), (2, 3), (2, 3), (4, 5), (4, 5),
                                            (6, 7), (6, 7)]
    for s in shards:
        assert s.num_q_heads == 4 and s.num_kv_heads == 1
        assert all(h // 8 == s.kv_start for h in range(s.q_start, s.q_stop))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_global_layer_up_to_four_ranks_needs_no_exchange(world):
    assert all(not head_shard(32, 4, world, r).shares_kv for r in range(world))


def test_uneven_splits_are_rejected():
    with pytest.raises(ValueError):
        head_shard(32, 4, 3, 0)
    with pytest.raises(ValueError):
        head_shard(12, 3, 2, 0)  # 6 query heads per rank straddle groups of 4
    with pytest.raises(ValueError):
        head_shard(12, 2, 3, 0)  # 4 query heads per rank cannot split a group of 6 evenly
    with pytest.raises(ValueError):
        head_shard(32, 4, 8, 8)


# ---------------------------------------------------------------- gloo ranks
def _oracle_fwd(q, k, v, *, window):
    o, lse = oracle.attention_fwd(q.numpy().transpose(0, 2, 1, 3), k.numpy().transpose(0, 2, 1, 3),
                                  v.numpy().transpose(0, 2, 1, 3), sliding_window=window or None,
                                  allow_vision_bidirectional=window > 0)
    return torch.from_numpy(o.transpose(0, 2, 1, 3).copy()), torch.from_numpy(lse)


def _oracle_bwd(q, k, v, out, lse, dout, *, window):
    t = lambda x: x.numpy().transpose(0, 2, 1, 3)  # noqa: E731
    dq, dk, dv = oracle.attention_bwd(t(q), t(k), t(v), t(dout), sliding_window=window or None,
                                      allow_vision_bidirectional=window > 0)
    back = lambda x: torch.from_numpy(x.transpose(0, 2, 1, 3).copy())  # noqa: E731
    return back(dq), back(dk), back(dv)


def _rank_main(rank, world, port, hq, hkv, window):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gemma4_fa4_kernels_b200.head_parallel import (HeadParallelGroup,
                                                           head_parallel_backward,
                                                           head_parallel_forward)

        g = torch.Generator().manual_seed(7)
        b, s, d = 2, 37, 16
        q = torch.randn(b, s, hq, d, generator=g, dtype=torch.float64)
        k = torch.randn(b, s, hkv, d, generator=g, dtype=torch.float64)
        v = torch.randn(b, s, hkv, d, generator=g, dtype=torch.float64)
        do = torch.randn(b, s, hq, d, generator=g, dtype=torch.float64)
        full_o, full_lse = _oracle_fwd(q, k, v, window=window)
        full_dq, full_dk, full_dv = _oracle_bwd(q, k, v, full_o, full_lse, do, window=window)

        hp = HeadParallelGroup(hq, hkv)
        lq, lk, lv = hp.local_heads(q, "q"), hp.local_heads(k, "kv"), hp.local_heads(v, "kv")
        ldo = hp.local_heads(do, "q")
        o, lse = head_parallel_forward(hp, lq, lk, lv, window=window, attn_fwd=_oracle_fwd)
        dq, dk, dv = head_parallel_backward(hp, lq, lk, lv, o, lse, ldo, window=window,
                                            attn_bwd=_oracle_bwd)
        sh = hp.shard
        np.testing.assert_allclose(o, full_o[:, :, sh.q_start:sh.q_stop], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(lse, full_lse[:, sh.q_start:sh.q_stop], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(dq, full_dq[:, :, sh.q_start:sh.q_stop], rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(dk, full_dk[:, :, sh.kv_start:sh.kv_stop], rtol=1e-10,
                                   atol=1e-10)
        np.testing.assert_allclose(dv, full_dv[:, :, sh.kv_start:sh.kv_stop], rtol=1e-10,
                                   atol=1e-10)
        # without the exchange, a shared KV head's gradient would be partial
        if sh.shares_kv:
            _, pk, _ = _oracle_bwd(lq, lk, lv, o, lse, ldo, window=window)
            assert not np.allclose(pk, full_dk[:, :, sh.kv_start:sh.kv_stop])

        # bench.py's multi-rank plumbing: barrier and max over ranks
        import bench

        bench.barrier(world)
        assert bench.max_over_ranks(float(rank + 1), world, torch.device("cpu")) == float(world)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hq,hkv,window", [(4, 1, 0), (4, 2, 0), (4, 1, 9), (8, 4, 9)],
                         ids=["shared-kv-global", "own-kv-global", "shared-kv-local",
                              "own-kv-local"])
def test_two_gloo_ranks_match_the_single_process_oracle(hq, hkv, window):
    mp.spawn(_rank_main, args=(2, _free_port(), hq, hkv, window), nprocs=2, join=True)
