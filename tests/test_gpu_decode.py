"""GPU parity of the single-token decode kernels (through the C ABI) against the oracle.

One query token per sequence at the lower-right position against a KV cache:
static-cache views with spare capacity (the layout the reference's decode ops
pass, h100_torch_ops.py:692-880), local windows shorter and longer than the
cache, documents, packed segments, and the split / merge path.
"""

import numpy as np
import pytest
import torch

import oracle
from parity_util import (LSE_ABS_TOL, REL_L2_TOL, bhsd_to_bshd, bshd_to_bhsd_np, lse_abs_err,
                         make_inputs, rel_l2, thd_np)

pytestmark = pytest.mark.gpu

cuda = pytest.importorskip("torch").cuda
if not cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib, ops  # noqa: E402


def _cache_view(x, capacity):
    """(B, L, H, D) values stored in a (B, H, capacity, D) static cache; returns
    the (B, L, H, D) view of the active prefix (token stride D, head stride
    capacity * D), as the reference builds it from StaticCache backings."""
    b, length, h, d = x.shape
    backing = torch.zeros(b, h, capacity, d, dtype=x.dtype, device=x.device)
    backing[:, :, :length] = x.transpose(1, 2)
    return backing[:, :, :length].transpose(1, 2)


def _decode_fixed(b, sk, hq, hkv, d, window, seed, capacity=None, docs=None):
    q, k, v = make_inputs((b, 1, hq, d), (b, sk, hkv, d), (b, sk, hkv, d), seed=seed,
                          with_dout=False)
    if capacity is not None:
        k = _cache_view(k, capacity)
        v = _cache_view(v, capacity)
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    before = _lib.launch_counts()
    out, lse = ops.attn_fwd(q, k, v, window=window, document_ids=doc_t)
    torch.cuda.synchronize()
    after = _lib.launch_counts()
    # sliding layers with query groups of at most 4 heads: the one-launch
    # short-window kernel; everything else the tensor-core split-key kernel
    kernel = "decode_short" if window > 0 and hq // hkv <= 4 else "decode"
    assert after[kernel] == before[kernel] + 1, f"{kernel} did not serve the call"
    if kernel == "decode_short":
        assert after["decode_combine"] == before["decode_combine"]  # merge fused
    ref_o, ref_lse = oracle.attention_fwd(
        bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
        sliding_window=window or None, allow_vision_bidirectional=window > 0,
        document_ids=None if docs is None else np.asarray(docs))
    e_o = rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o))
    e_l = lse_abs_err(lse.cpu().numpy(), ref_lse)
    assert e_o <= REL_L2_TOL, f"O rel-L2 {e_o:.3e}"
    assert e_l <= LSE_ABS_TOL, f"LSE abs {e_l:.3e}"
    return out, lse, after["decode_combine"] - before["decode_combine"]


@pytest.mark.parametrize("sk", [1, 100, 128, 129, 1000, 4097])
def test_global_d512_decode_static_cache(sk):
    _decode_fixed(1, sk, 32, 4, 512, 0, seed=sk, capacity=sk + 37)


def test_global_d512_decode_splits_and_merges():
    # 2 x 1 KV units -> many key splits per unit, merged by the combine kernel.
    _, _, merges = _decode_fixed(2, 5000, 8, 1, 512, 0, seed=5)
    assert merges == 1


@pytest.mark.parametrize("sk", [1, 300, 1024, 1025, 3000])
def test_local_d256_decode_window(sk):
    # window 1024: a longer cache keeps only the last 1024 keys
    _decode_fixed(1, sk, 32, 16, 256, 1024, seed=50 + sk, capacity=max(sk, 1024))


@pytest.mark.parametrize("b,hq,hkv,d,sk", [(1, 32, 16, 256, 1024), (3, 8, 2, 512, 700),
                                            (2, 4, 4, 256, 97)],
                         ids=["c4_local_window", "d512_group4", "group1"])
def test_short_window_decode_shapes(b, hq, hkv, d, sk):
    """The short-window kernel over its template range (head dims, groups of
    1-4 query heads) with several splits merged by the last arriving CTA."""
    _decode_fixed(b, sk, hq, hkv, d, 1024, seed=80 + sk, capacity=sk + 64)


def test_short_window_decode_repeats_on_one_workspace():
    """The merge counters return to zero after every call: repeated calls on
    the same inputs give identical results."""
    q, k, v = make_inputs((1, 1, 32, 256), (1, 1024, 16, 256), (1, 1024, 16, 256), seed=88,
                          with_dout=False)
    o1, l1 = ops.attn_fwd(q, k, v, window=1024)
    for _ in range(3):
        o2, l2 = ops.attn_fwd(q, k, v, window=1024)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_local_d256_decode_documents():
    sk = 900
    docs = np.zeros((2, sk), dtype=np.int32)
    docs[0, 400:] = 1
    docs[1, 10:] = 3
    docs[1, 899:] = 4  # the query's document holds only itself
    _decode_fixed(2, sk, 4, 2, 256, 1024, seed=61, docs=docs)


def test_decode_matches_full_prefill_last_row():
    # The decode path and the prefill path agree on the last query row.
    s = 700
    q, k, v = make_inputs((1, s, 8, 512), (1, s, 1, 512), (1, s, 1, 512), seed=71,
                          with_dout=False)
    o_full, l_full = ops.attn_fwd(q, k, v, window=0)
    o_dec, l_dec = ops.attn_fwd(q[:, -1:].contiguous(), k, v, window=0)
    torch.cuda.synchronize()
    assert rel_l2(o_dec.float().cpu().numpy(), o_full[:, -1:].float().cpu().numpy()) < 1e-2
    assert (l_dec[..., 0] - l_full[..., -1]).abs().max().item() < 1e-3


def test_decode_is_bit_deterministic():
    q, k, v = make_inputs((1, 1, 32, 512), (1, 3000, 4, 512), (1, 3000, 4, 512), seed=72,
                          with_dout=False)
    o1, l1 = ops.attn_fwd(q, k, v, window=0)
    o2, l2 = ops.attn_fwd(q, k, v, window=0)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


@pytest.mark.parametrize("d,hq,hkv,window", [(512, 8, 1, 0), (256, 4, 2, 1024)])
def test_packed_decode_segments(d, hq, hkv, window):
    cu_q = [0, 1, 1, 2, 3, 4]          # segment 1 has no query token
    lk = [5, 40, 1300, 128, 2100]
    cu_k = np.concatenate([[0], np.cumsum(lk)]).tolist()
    tq, tk = cu_q[-1], cu_k[-1]
    q, k, v = make_inputs((tq, hq, d), (tk, hkv, d), (tk, hkv, d), seed=81 + d, with_dout=False)
    docs = None
    if window:
        docs = np.zeros(tk, dtype=np.int32)
        docs[cu_k[3] + 60:cu_k[4]] = 2  # segment 3: query in a later document
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    out, lse = ops.attn_fwd(q, k, v, window=window, cu_seqlens_q=cq, cu_seqlens_k=ck,
                            max_seqlen_q=1, max_seqlen_k=max(lk), document_ids=doc_t)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle.attention_fwd_varlen(
        thd_np(q), thd_np(k), thd_np(v), cu_q, cu_k, sliding_window=window or None,
        allow_vision_bidirectional=window > 0, document_ids=docs)
    assert rel_l2(out.float().cpu().numpy(), ref_o) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL


def test_global_forward_only_adapter_runs_decode():
    from gemma4_fa4_kernels_b200 import fa4_global_forward_only

    sk = 2500
    q, k, v = make_inputs((1, 1, 32, 512), (1, sk, 4, 512), (1, sk, 4, 512), seed=91,
                          with_dout=False)
    k = _cache_view(k, 4096)
    v = _cache_view(v, 4096)
    before = _lib.launch_counts()["decode"]
    out, lse = fa4_global_forward_only(q, k, v)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["decode"] == before + 1
    ref_o, ref_lse = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k),
                                          bshd_to_bhsd_np(v))
    assert rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o)) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL


def test_decode_rescales_when_the_running_max_jumps():
    # Growing keys move every head's running max far past the lazy-rescale
    # threshold from one key split / tile to the next.
    sk = 3000
    q, k, v = make_inputs((1, 1, 8, 512), (1, sk, 1, 512), (1, sk, 1, 512), seed=93,
                          with_dout=False)
    ramp = torch.linspace(0.1, 8.0, sk, device="cuda").view(1, sk, 1, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    q = (q.float() + 0.5 * k.float().mean(dim=1, keepdim=True).expand_as(q)).to(torch.bfloat16)
    out, lse = ops.attn_fwd(q, k, v, window=0)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k),
                                          bshd_to_bhsd_np(v))
    assert rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o)) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL
