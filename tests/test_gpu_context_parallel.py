"""Context parallelism on the GPU: the ring merge / cast / add kernels, a
one-rank ring (its two diagonal blocks through the kernels), and, on a box with
two or more GPUs, two NCCL ranks running the full ring (global d512) and the
halo exchange (local d256) against the float64 oracle and the one-GPU call.

Multi-rank cases spawn child processes, one per GPU, with NCCL's NVLink
multicast (NVLS) off and a short process-group timeout."""

import os
import socket

import numpy as np
import pytest
import torch

from parity_util import (LSE_ABS_TOL, REL_L2_TOL, bshd_to_bhsd_np, lse_abs_err, make_inputs,
                         rel_l2)

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import oracle  # noqa: E402
from gemma4_fa4_kernels_b200 import ops  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_merge_cast_and_add_kernels():
    g = torch.Generator().manual_seed(1)
    t, h, d = 300, 4, 512
    o_acc = torch.randn(1, t, h, d, generator=g)
    lse_acc = torch.randn(1, h, t, generator=g) * 3
    o_part = torch.randn(1, t, h, d, generator=g).to(torch.bfloat16)
    lse_part = torch.randn(1, h, t, generator=g) * 3
    lse_acc[0, 0, :7] = float("-inf")   # rows not reached yet
    lse_part[0, 1, :5] = float("-inf")  # a block that masks its rows
    lse_acc[0, 2, :3] = lse_part[0, 2, :3] = float("-inf")  # neither
    o_acc[0, :3, 2] = 0
    oa, la = o_acc.double(), lse_acc.double()
    ob, lb = o_part.double(), lse_part.double()
    lse_ref = torch.logaddexp(la, lb)
    wa = torch.where(torch.isfinite(lse_ref), torch.exp(la - lse_ref), torch.ones_like(la))
    wb = torch.where(torch.isfinite(lse_ref), torch.exp(lb - lse_ref), torch.zeros_like(lb))
    o_ref = oa * wa[0].T[None, ..., None] + ob * wb[0].T[None, ..., None]
    dev_o, dev_l = o_acc.cuda(), lse_acc.cuda()
    ops.merge_partial(dev_o, dev_l, o_part.cuda(), lse_part.cuda())
    torch.cuda.synchronize()
    assert torch.allclose(dev_o.cpu().double(), o_ref, rtol=1e-5, atol=1e-5)
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(dev_l.cpu()), fin)
    assert torch.allclose(dev_l.cpu().double()[fin], lse_ref[fin], atol=1e-5)
    cast = ops.cast_f32_bf16(dev_o)
    assert torch.equal(cast.cpu(), dev_o.cpu().to(torch.bfloat16))
    x, y = torch.randn(1000, generator=g).cuda(), torch.randn(1000, generator=g).cuda()
    ref = (x + y).cpu()
    ops.add_f32_(x, y)
    assert torch.equal(x.cpu(), ref)


def test_one_rank_ring_matches_the_oracle():
    """World size 1: the ring reduces to its two diagonal blocks (causal and
    rectangular lower-right), merged from an empty accumulator."""
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0,
                            world_size=1)
    try:
        _one_rank_ring()
    finally:
        dist.destroy_process_group()


def _one_rank_ring():
    from gemma4_fa4_kernels_b200.context_parallel import ring_global_attention

    s, hq, hkv, d = 1400, 8, 1, 512
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=21)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, lse = ring_global_attention(qd, kd, vd)
    out.backward(do)
    torch.cuda.synchronize()
    qn, kn, vn, don = (bshd_to_bhsd_np(t) for t in (q, k, v, do))
    ro, rl = oracle.attention_fwd(qn, kn, vn)
    rq, rk, rv = oracle.attention_bwd(qn, kn, vn, don)
    assert rel_l2(bshd_to_bhsd_np(out), ro) <= REL_L2_TOL
    assert lse_abs_err(lse.detach().cpu().numpy(), rl) <= LSE_ABS_TOL
    for g, r in ((qd.grad, rq), (kd.grad, rk), (vd.grad, rv)):
        assert rel_l2(bshd_to_bhsd_np(g), r) <= REL_L2_TOL


def _rank_main(rank, world, port, kind):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from gemma4_fa4_kernels_b200.context_parallel import (halo_local_backward,
                                                              halo_local_forward,
                                                              ring_global_attention,
                                                              zigzag_shard)

        if kind == "ring":
            s, hq, hkv, d = 2 * world * 600, 8, 1, 512
            q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=22,
                                      device="cpu")
            sh = lambda x: zigzag_shard(x, rank, world).to(dev)  # noqa: E731
            qd, kd, vd = (sh(t).requires_grad_(True) for t in (q, k, v))
            out, lse = ring_global_attention(qd, kd, vd)
            out.backward(sh(do))
            torch.cuda.synchronize()
            qn, kn, vn, don = (bshd_to_bhsd_np(t) for t in (q, k, v, do))
            ro, rl = oracle.attention_fwd(qn, kn, vn)
            rq, rk, rv = oracle.attention_bwd(qn, kn, vn, don)
            back = lambda x: torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3)))  # noqa
            shn = lambda x: bshd_to_bhsd_np(zigzag_shard(back(x), rank, world))  # noqa: E731
            assert rel_l2(bshd_to_bhsd_np(out), shn(ro)) <= REL_L2_TOL
            rl_sh = zigzag_shard(torch.from_numpy(rl), rank, world, dim=2).numpy()
            assert lse_abs_err(lse.detach().cpu().numpy(), rl_sh) <= LSE_ABS_TOL
            for g, r in ((qd.grad, rq), (kd.grad, rk), (vd.grad, rv)):
                assert rel_l2(bshd_to_bhsd_np(g), shn(r)) <= REL_L2_TOL
        else:
            w, c, hq, hkv, d = 1024, 1500, 4, 2, 256
            s = world * c
            q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=23,
                                      device="cpu")
            vis = torch.full((s,), -1, dtype=torch.int32)
            vis[200:456] = 0
            vis[c + 300:c + 556] = 1
            rows = slice(rank * c, (rank + 1) * c)
            loc = lambda x: x[:, rows].contiguous().to(dev)  # noqa: E731
            out, lse = halo_local_forward(loc(q), loc(k), loc(v), window=w,
                                          vision_ids=vis.to(dev))
            dq, dk, dv = halo_local_backward(loc(q), loc(k), loc(v), out, lse, loc(do), window=w,
                                             vision_ids=vis.to(dev))
            torch.cuda.synchronize()
            qn, kn, vn, don = (bshd_to_bhsd_np(t) for t in (q, k, v, do))
            kw = dict(sliding_window=w, allow_vision_bidirectional=True,
                      vision_block_ids=vis.numpy()[None])
            ro, rl = oracle.attention_fwd(qn, kn, vn, **kw)
            rq, rk, rv = oracle.attention_bwd(qn, kn, vn, don, **kw)
            assert rel_l2(bshd_to_bhsd_np(out), ro[:, :, rows]) <= REL_L2_TOL
            assert lse_abs_err(lse.cpu().numpy(), rl[:, :, rows]) <= LSE_ABS_TOL
            for g, r in ((dq, rq), (dk, rk), (dv, rv)):
                assert rel_l2(bshd_to_bhsd_np(g), r[:, :, rows]) <= REL_L2_TOL
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kind", ["ring", "halo"])
def test_two_nccl_ranks_match_the_oracle(kind):
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port(), kind), nprocs=2, join=True)
