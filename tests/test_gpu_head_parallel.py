"""Head-parallel attention on 2 GPUs (NCCL): each rank runs the CUDA kernels on
its query heads; ranks sharing a KV head sum their dK/dV.  Compared against
the full single-GPU call.  Skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs 2 CUDA devices", allow_module_level=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-6)).item()


def _rank_main(rank, world, port, hq, hkv, d, window):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from gemma4_fa4_kernels_b200 import ops
        from gemma4_fa4_kernels_b200.head_parallel import (HeadParallelGroup,
                                                           head_parallel_backward,
                                                           head_parallel_forward)

        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(11)
        s = 700

        def rms(x):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

        q = rms(torch.randn(1, s, hq, d, generator=g)).bfloat16().to(dev)
        k = rms(torch.randn(1, s, hkv, d, generator=g)).bfloat16().to(dev)
        v = rms(torch.randn(1, s, hkv, d, generator=g)).bfloat16().to(dev)
        do = torch.randn(1, s, hq, d, generator=g).bfloat16().to(dev)
        full_o, full_lse = ops.attn_fwd(q, k, v, window=window)
        full_dq, full_dk, full_dv = ops.attn_bwd(q, k, v, full_o, full_lse, do, window=window)

        hp = HeadParallelGroup(hq, hkv)
        sh = hp.shard
        lq = hp.local_heads(q, "q").contiguous()
        lk = hp.local_heads(k, "kv").contiguous()
        lv = hp.local_heads(v, "kv").contiguous()
        ldo = hp.local_heads(do, "q").contiguous()
        o, lse = head_parallel_forward(hp, lq, lk, lv, window=window)
        dq, dk, dv = head_parallel_backward(hp, lq, lk, lv, o, lse, ldo, window=window)
        torch.cuda.synchronize(dev)
        # forward and dQ of a head do not depend on the other heads: bit-identical
        assert torch.equal(o, full_o[:, :, sh.q_start:sh.q_stop])
        assert torch.equal(lse, full_lse[:, sh.q_start:sh.q_stop])
        assert torch.equal(dq, full_dq[:, :, sh.q_start:sh.q_stop])
        # dK/dV: partial sums rounded to BF16 once more when shared
        assert _rel(dk, full_dk[:, :, sh.kv_start:sh.kv_stop]) < 1e-2
        assert _rel(dv, full_dv[:, :, sh.kv_start:sh.kv_stop]) < 1e-2
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("hq,hkv,d,window", [(8, 1, 512, 0), (8, 4, 256, 1024)],
                         ids=["global-shared-kv", "local-own-kv"])
def test_two_gpu_head_parallel_matches_single_gpu(hq, hkv, d, window):
    mp.spawn(_rank_main, args=(2, _free_port(), hq, hkv, d, window), nprocs=2, join=True)
