"""GPU tests of the reference-facing adapters (autograd included), the CUDA mask
builder and the reference's sentinel / known-answer cases (through the C ABI)."""

import json
import os

import numpy as np
import pytest
import torch

import oracle
from parity_util import (LSE_ABS_TOL, assert_close_to_oracle, bhsd_to_bshd, bshd_to_bhsd_np,
                         lse_abs_err, make_inputs, thd_np)

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gemma4_fa4_kernels_b200 as g4  # noqa: E402
from gemma4_fa4_kernels_b200 import GLOBAL_ATTENTION, SLIDING_ATTENTION  # noqa: E402

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "masks.json")


def _grad_case(fn, spec, s, seed, *, vision=None, with_dlse=False):
    q, k, v, do = make_inputs((1, s, spec.num_q_heads, spec.head_dim_qk),
                              (1, s, spec.num_kv_heads, spec.head_dim_qk),
                              (1, s, spec.num_kv_heads, spec.head_dim_v), seed=seed)
    dlse = torch.randn(1, spec.num_q_heads, s, device="cuda") if with_dlse else None
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    kw = {} if vision is None else {"vision_block_ids": torch.tensor(vision, device="cuda")}
    out, lse = fn(qd, kd, vd, **kw)
    loss = (out.float() * do.float()).sum()
    if dlse is not None:
        loss = loss + (lse * dlse).sum()
    loss.backward()
    torch.cuda.synchronize()
    okw = dict(sliding_window=spec.sliding_window,
               allow_vision_bidirectional=spec.sliding_window is not None,
               vision_block_ids=None if vision is None else np.asarray(vision))
    ro, rl = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v), **okw)
    rq, rk, rv = oracle.attention_bwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
                                      bshd_to_bhsd_np(do),
                                      dlse=None if dlse is None else dlse.double().cpu().numpy(),
                                      **okw)
    assert_close_to_oracle("out", bshd_to_bhsd_np(out), ro)
    assert lse_abs_err(lse.detach().cpu().numpy(), rl) <= LSE_ABS_TOL
    for name, got, ref in (("dq", qd.grad, rq), ("dk", kd.grad, rk), ("dv", vd.grad, rv)):
        assert_close_to_oracle(name, bshd_to_bhsd_np(got), ref)


def test_local_text_adapter_autograd_full_heads():
    _grad_case(g4.fa4_local_text_forward, SLIDING_ATTENTION, 300, seed=1)


def test_local_vision_adapter_autograd():
    s = 320
    vision = np.full((1, s), -1, dtype=np.int64)
    vision[0, 40:140] = 0
    vision[0, 200:260] = 3
    _grad_case(g4.fa4_local_forward, SLIDING_ATTENTION, s, seed=2, vision=vision)


def test_global_text_adapter_autograd_with_lse_gradient():
    _grad_case(g4.fa4_global_text_forward, GLOBAL_ATTENTION, 200, seed=3, with_dlse=True)


def test_global_lse_only_gradient_gives_exact_zero_dv():
    # reference probe policy: an LSE-only upstream gradient yields exact-zero dV
    spec = GLOBAL_ATTENTION
    q, k, v, _ = make_inputs((1, 150, 32, 512), (1, 150, 4, 512), (1, 150, 4, 512), seed=4)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    _out, lse = g4.fa4_global_text_forward(qd, kd, vd, spec=spec)
    lse.sum().backward()
    torch.cuda.synchronize()
    assert torch.count_nonzero(vd.grad) == 0
    assert torch.count_nonzero(qd.grad) > 0


def test_global_forward_only_rectangular_batched():
    q, k, v, _ = make_inputs((2, 70, 32, 512), (2, 190, 4, 512), (2, 190, 4, 512), seed=5)
    out, lse = g4.fa4_global_forward_only(q, k, v)
    torch.cuda.synchronize()
    ro, rl = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v))
    assert_close_to_oracle("out", bshd_to_bhsd_np(out), ro)
    assert lse_abs_err(lse.detach().cpu().numpy(), rl) <= LSE_ABS_TOL


def test_local_varlen_adapter_metadata_autograd():
    spec = SLIDING_ATTENTION
    cu = [0, 150, 150, 420]
    t = cu[-1]
    q, k, v, do = make_inputs((t, 32, 256), (t, 16, 256), (t, 16, 256), seed=6)
    vision = torch.full((t,), -1, dtype=torch.int32)
    vision[20:90] = 1
    vision[300:380] = 1
    docs = torch.zeros(t, dtype=torch.int32)
    docs[350:] = 4
    cq = torch.tensor(cu, dtype=torch.int32, device="cuda")
    qd, kd, vd = (x.clone().requires_grad_(True) for x in (q, k, v))
    out, lse = g4.fa4_local_varlen_forward(qd, kd, vd, cq, cq, max_seqlen_q=270, max_seqlen_k=270,
                                           vision_block_ids=vision.cuda(),
                                           document_ids=docs.cuda(), spec=spec)
    out.backward(do)
    torch.cuda.synchronize()
    ro, rl, rq, rk, rv = oracle.attention_fwd_bwd_varlen(
        thd_np(q), thd_np(k), thd_np(v), thd_np(do), cu, cu, sliding_window=1024,
        vision_block_ids=vision.numpy(), document_ids=docs.numpy(), allow_vision_bidirectional=True)
    assert_close_to_oracle("out", thd_np(out), ro)
    assert lse_abs_err(lse.detach().cpu().numpy(), rl) <= LSE_ABS_TOL
    for name, got, ref in (("dq", qd.grad, rq), ("dk", kd.grad, rk), ("dv", vd.grad, rv)):
        assert_close_to_oracle(name, thd_np(got), ref)


def test_global_varlen_adapters():
    cu_q, cu_k = [0, 3, 3, 200], [0, 10, 12, 300]
    q, k, v, do = make_inputs((200, 32, 512), (300, 4, 512), (300, 4, 512), seed=7)
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    with torch.no_grad():
        o1, l1 = g4.fa4_global_varlen_forward_only(q, k, v, cq, ck, max_seqlen_q=197,
                                                   max_seqlen_k=288)
    qd, kd, vd = (x.clone().requires_grad_(True) for x in (q, k, v))
    o2, l2 = g4.fa4_global_varlen_forward(qd, kd, vd, cq, ck, max_seqlen_q=197, max_seqlen_k=288)
    o2.backward(do)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    ro, rl, rq, rk, rv = oracle.attention_fwd_bwd_varlen(thd_np(q), thd_np(k), thd_np(v),
                                                         thd_np(do), cu_q, cu_k)
    assert_close_to_oracle("out", thd_np(o2), ro)
    for name, got, ref in (("dq", qd.grad, rq), ("dk", kd.grad, rk), ("dv", vd.grad, rv)):
        assert_close_to_oracle(name, thd_np(got), ref)
    # keys of the empty-query segment receive exact zeros
    assert torch.count_nonzero(kd.grad[10:12]) == 0 and torch.count_nonzero(vd.grad[10:12]) == 0


def test_cuda_mask_builder_matches_reference_golden():
    cases = json.load(open(GOLD))
    for name, c in cases.items():
        t = lambda x, dt: None if x is None else torch.tensor(x, dtype=dt)  # noqa: E731
        m = g4.gemma4_attention_mask(
            batch_size=c["b"], q_len=c["q_len"], kv_len=c["kv_len"], device="cuda",
            sliding_window=c["window"], vision_block_ids=t(c["vision"], torch.int32),
            document_ids=t(c["docs"], torch.int32), key_padding_mask=t(c["padding"], torch.bool),
            allow_vision_bidirectional=c["bidir"])
        want = np.asarray(c["mask"], np.uint8).reshape(c["shape"])
        np.testing.assert_array_equal(m.cpu().numpy().astype(np.uint8), want, err_msg=name)


def test_masked_kv_sentinels_do_not_leak():
    # reference test_h100_fa4.py:2079-2115: a masked future key with huge K/V
    # values must not change the query's output or LSE bit for bit.
    seqlen, query, allowed_future, masked_future = 65, 31, 32, 33
    q = torch.zeros(1, seqlen, 32, 256, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, seqlen, 16, 256, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, seqlen, 16, 256, device="cuda").to(torch.bfloat16)
    ids = torch.full((1, seqlen), -1, device="cuda", dtype=torch.int32)
    ids[:, query:allowed_future + 1] = 0
    ids[:, masked_future] = 1
    q[:, query, 0, 0] = 1
    o0, l0 = g4.fa4_local_forward(q, k, v, vision_block_ids=ids)
    km, vm = k.clone(), v.clone()
    km[:, masked_future, 0, 0] = 128
    vm[:, masked_future, 0] = 128
    o1, l1 = g4.fa4_local_forward(q, km, vm, vision_block_ids=ids)
    assert torch.equal(o1[:, query, 0], o0[:, query, 0])
    assert torch.equal(l1[:, 0, query], l0[:, 0, query])
    va = v.clone()
    va[:, allowed_future, 0] = 128
    o2, _ = g4.fa4_local_forward(q, k, va, vision_block_ids=ids)
    assert not torch.equal(o2[:, query, 0], o0[:, query, 0])


def test_strict_w1024_window_edge_sentinel():
    # reference test_h100_fa4.py:1934-1976 (the W1024 known answer on device)
    q = torch.zeros(1, 32, 256, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1025, 16, 256, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    cu_q = torch.tensor([0, 1], device="cuda", dtype=torch.int32)
    cu_k = torch.tensor([0, 1025], device="cuda", dtype=torch.int32)
    ids = torch.zeros(1025, device="cuda", dtype=torch.int32)
    v_ex = v.clone()
    v_ex[0, 0] = 2048
    o_ex, l_ex = g4.fa4_local_varlen_forward(q, k, v_ex, cu_q, cu_k, max_seqlen_q=1,
                                             max_seqlen_k=1025, vision_block_ids=ids)
    assert torch.count_nonzero(o_ex[0, 0]) == 0
    v_in = v.clone()
    v_in[1, 0] = 2048
    o_in, l_in = g4.fa4_local_varlen_forward(q, k, v_in, cu_q, cu_k, max_seqlen_q=1,
                                             max_seqlen_k=1025, vision_block_ids=ids)
    assert torch.equal(o_in[0, 0], torch.full_like(o_in[0, 0], 2.0))
    assert torch.equal(l_in, l_ex)


def test_head_partition_shares_match_the_full_call():
    # Query heads with their KV group split over 8 ranks (run here one share at
    # a time) reproduce the full-model forward bit for bit.
    spec = SLIDING_ATTENTION
    q, k, v, _ = make_inputs((1, 260, 32, 256), (1, 260, 16, 256), (1, 260, 16, 256), seed=9)
    full, lse = g4.fa4_local_text_forward(q, k, v)
    for r in range(8):
        part = spec.head_partition(8, r)
        qs = q[:, :, 4 * r:4 * r + 4].contiguous()
        ks = k[:, :, 2 * r:2 * r + 2].contiguous()
        vs = v[:, :, 2 * r:2 * r + 2].contiguous()
        o, l_ = g4.fa4_local_text_forward(qs, ks, vs, spec=part)
        assert torch.equal(o, full[:, :, 4 * r:4 * r + 4])
        assert torch.equal(l_, lse[:, 4 * r:4 * r + 4])
