"""GPU parity of the backward kernels (through the C ABI) against the oracle."""

import numpy as np
import pytest
import torch

import oracle
from parity_util import (assert_close_to_oracle, bhsd_to_bshd, bshd_to_bhsd_np,
                         eager_bf16_attention, make_inputs, thd_np)

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import ops  # noqa: E402


def _fixed(b, sq, sk, hq, hkv, d, window, seed, vision=None, docs=None, with_dlse=False,
           check_eager=True):
    ins = make_inputs((b, sq, hq, d), (b, sk, hkv, d), (b, sk, hkv, d), seed=seed,
                      dlse_shape=(b, hq, sq) if with_dlse else None)
    q, k, v, dout = ins[:4]
    dlse = ins[4] if with_dlse else None
    vis_t = None if vision is None else torch.tensor(vision, dtype=torch.int32, device="cuda")
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    out, lse = ops.attn_fwd(q, k, v, window=window, vision_ids=vis_t, document_ids=doc_t)
    dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, dout, dlse=dlse, window=window,
                              vision_ids=vis_t, document_ids=doc_t)
    torch.cuda.synchronize()
    kw = dict(sliding_window=window or None, allow_vision_bidirectional=window > 0,
              vision_block_ids=None if vision is None else np.asarray(vision),
              document_ids=None if docs is None else np.asarray(docs))
    rq, rk, rv = oracle.attention_bwd(
        bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v), bshd_to_bhsd_np(dout),
        dlse=None if dlse is None else dlse.double().cpu().numpy(), **kw)
    eager = [None] * 3
    if check_eager and dlse is None:
        mask = oracle.gemma4_attention_mask(batch_size=b, q_len=sq, kv_len=sk,
                                            sliding_window=kw["sliding_window"],
                                            vision_block_ids=kw["vision_block_ids"],
                                            document_ids=kw["document_ids"],
                                            allow_vision_bidirectional=window > 0)
        allowed = torch.from_numpy(mask).to("cuda")
        _, grads = eager_bf16_attention(q, k, v, allowed, dout)
        eager = [bshd_to_bhsd_np(g) for g in grads]
    for name, got, ref, eg in (("dq", dq, rq, eager[0]), ("dk", dk, rk, eager[1]),
                               ("dv", dv, rv, eager[2])):
        assert_close_to_oracle(name, bshd_to_bhsd_np(got), ref, eg)
    return dq, dk, dv


@pytest.mark.parametrize("s", [1, 100, 128, 300, 1100])
def test_local_d256_text_fixed(s):
    _fixed(1, s, s, 4, 2, 256, 1024, seed=200 + s)


@pytest.mark.parametrize("hq,hkv", [(2, 2), (6, 2), (8, 2)], ids=["g1", "g3", "g4"])
def test_local_d256_group_sizes(hq, hkv):
    """Query groups of 1, 3 and 4 heads per KV head: the persistent forward's
    KV-head mapping, and dQ with head pairs per CTA (even groups) or one head
    per CTA (odd groups)."""
    _fixed(1, 700, 700, hq, hkv, 256, 1024, seed=210 + hq)


@pytest.mark.parametrize("s", [1, 130, 400])
def test_global_d512_causal_fixed(s):
    _fixed(1, s, s, 8, 1, 512, 0, seed=300 + s)


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (6, 2)], ids=["g1", "g2", "g3"])
def test_global_d512_group_sizes(hq, hkv):
    """Query groups of 1, 2 and 3 heads per KV head at d512: the dQ GEMM runs
    as 2-CTA pairs over heads 2i, 2i+1 of a group for even groups, one CTA per
    head otherwise, and dK / dV sum every group size in TMEM."""
    _fixed(1, 300, 300, hq, hkv, 512, 0, seed=220 + hq)


def test_global_d512_rectangular_with_dlse():
    _fixed(1, 90, 260, 8, 1, 512, 0, seed=41, with_dlse=True)


def test_local_d256_dlse_small_window():
    _fixed(2, 260, 260, 4, 2, 256, 77, seed=42, with_dlse=True)


def test_local_d256_vision_and_documents():
    s = 600
    vision = np.full((1, s), -1, dtype=np.int32)
    vision[0, 100:230] = 1
    vision[0, 300:380] = 2
    vision[0, 520:560] = 1   # same id later, non-contiguous
    docs = np.zeros((1, s), dtype=np.int32)
    docs[0, 450:] = 3
    _fixed(1, s, s, 4, 2, 256, 1024, seed=43, vision=vision, docs=docs)


def _packed(cu_q, cu_k, hq, hkv, d, window, seed, vision=None, docs=None):
    tq, tk = cu_q[-1], cu_k[-1]
    q, k, v, dout = make_inputs((tq, hq, d), (tk, hkv, d), (tk, hkv, d), seed=seed)
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    mq, mk = int(np.diff(cu_q).max()), int(np.diff(cu_k).max())
    vis_t = None if vision is None else torch.tensor(vision, dtype=torch.int32, device="cuda")
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    kw = dict(window=window, cu_seqlens_q=cq, cu_seqlens_k=ck, max_seqlen_q=mq, max_seqlen_k=mk,
              vision_ids=vis_t, document_ids=doc_t)
    out, lse = ops.attn_fwd(q, k, v, **kw)
    dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, dout, **kw)
    torch.cuda.synchronize()
    _, _, rq, rk, rv = oracle.attention_fwd_bwd_varlen(
        thd_np(q), thd_np(k), thd_np(v), thd_np(dout), cu_q, cu_k,
        sliding_window=window or None, allow_vision_bidirectional=window > 0,
        vision_block_ids=vision, document_ids=docs)
    for name, got, ref in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert_close_to_oracle(name, thd_np(got), ref)
    # keys of segments with no queries get exact zeros
    for s0, s1, e0, e1 in zip(cu_q[:-1], cu_q[1:], cu_k[:-1], cu_k[1:]):
        if s1 == s0:
            assert torch.count_nonzero(dk[e0:e1]) == 0 and torch.count_nonzero(dv[e0:e1]) == 0


def test_local_d256_packed_mixed_empty():
    _packed([0, 100, 100, 400, 1500], [0, 130, 200, 600, 1800], 4, 2, 256, 1024, seed=51)


def test_global_d512_packed():
    _packed([0, 5, 300, 301, 650], [0, 5, 300, 302, 800], 8, 1, 512, 0, seed=52)


def test_local_d256_packed_vision_documents():
    cu = [0, 300, 800, 1200]
    t = cu[-1]
    vision = np.full(t, -1, dtype=np.int32)
    vision[50:180] = 2
    vision[400:656] = 0
    vision[900:1000] = 0
    docs = np.zeros(t, dtype=np.int32)
    docs[600:] = 1
    docs[1100:] = 2
    _packed(cu, cu, 4, 2, 256, 1024, seed=53, vision=vision, docs=docs)


def test_backward_is_deterministic():
    q, k, v, dout = make_inputs((1, 500, 8, 512), (1, 500, 1, 512), (1, 500, 1, 512), seed=61)
    out, lse = ops.attn_fwd(q, k, v, window=0)
    g1 = ops.attn_bwd(q, k, v, out, lse, dout, window=0)
    g2 = ops.attn_bwd(q, k, v, out, lse, dout, window=0)
    torch.cuda.synchronize()
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


@pytest.mark.parametrize("shape", [(1, 300, 4, 2, 256, 1024), (1, 260, 8, 1, 512, 0)],
                         ids=["local_d256", "global_d512"])
def test_recompute_and_materialized_backward_agree_with_oracle(shape):
    b, s, hq, hkv, d, window = shape
    q, k, v, dout = make_inputs((b, s, hq, d), (b, s, hkv, d), (b, s, hkv, d), seed=71)
    out, lse = ops.attn_fwd(q, k, v, window=window)
    rq, rk, rv = oracle.attention_bwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
                                      bshd_to_bhsd_np(dout), sliding_window=window or None,
                                      allow_vision_bidirectional=window > 0)
    for algo in ("recompute", "materialized"):
        dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, dout, window=window, algorithm=algo)
        torch.cuda.synchronize()
        for name, got, ref in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
            assert_close_to_oracle(f"{algo} {name}", bshd_to_bhsd_np(got), ref)


@pytest.mark.parametrize("d,hq,hkv,window", [(512, 8, 1, 0), (256, 4, 2, 1024)])
def test_forward_backward_capture_into_a_cuda_graph(d, hq, hkv, window):
    # The backward forks its preprocessing onto a second stream and joins it
    # with events; the whole step must capture into a graph and replay with
    # results bit-identical to eager calls.
    s = 640
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=123)
    o_ref, l_ref = ops.attn_fwd(q, k, v, window=window)
    dq_ref, dk_ref, dv_ref = ops.attn_bwd(q, k, v, o_ref, l_ref, do, window=window)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):  # warm-up outside capture (allocator, attributes)
        o, l_ = ops.attn_fwd(q, k, v, window=window)
        ops.attn_bwd(q, k, v, o, l_, do, window=window)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o_g, l_g = ops.attn_fwd(q, k, v, window=window)
        dq_g, dk_g, dv_g = ops.attn_bwd(q, k, v, o_g, l_g, do, window=window)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(o_g, o_ref) and torch.equal(l_g, l_ref)
    assert torch.equal(dq_g, dq_ref) and torch.equal(dk_g, dk_ref) and torch.equal(dv_g, dv_ref)
