"""GPU parity of the forward kernel (through the C ABI) against the oracle."""

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

from gemma4_fa4_kernels_b200 import ops  # noqa: E402


def _fixed_case(b, sq, sk, hq, hkv, d, window, seed, vision=None, docs=None):
    q, k, v = make_inputs((b, sq, hq, d), (b, sk, hkv, d), (b, sk, hkv, d), seed=seed,
                          with_dout=False)
    vis_t = None if vision is None else torch.tensor(vision, dtype=torch.int32, device="cuda")
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    out, lse = ops.attn_fwd(q, k, v, window=window, vision_ids=vis_t, document_ids=doc_t)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle.attention_fwd(
        bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
        sliding_window=window or None, allow_vision_bidirectional=window > 0,
        vision_block_ids=None if vision is None else np.asarray(vision),
        document_ids=None if docs is None else np.asarray(docs))
    e_o = rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o))
    e_l = lse_abs_err(lse.cpu().numpy(), ref_lse)
    assert e_o <= REL_L2_TOL, f"O rel-L2 {e_o:.3e}"
    assert e_l <= LSE_ABS_TOL, f"LSE abs {e_l:.3e}"
    return out, lse


@pytest.mark.parametrize("s", [1, 63, 128, 129, 300, 1025, 2048])
def test_local_d256_text_fixed(s):
    _fixed_case(1, s, s, 4, 2, 256, 1024, seed=s)


@pytest.mark.parametrize("s", [1, 65, 257, 640])
def test_global_d512_causal_fixed(s):
    _fixed_case(1, s, s, 8, 1, 512, 0, seed=100 + s)


@pytest.mark.parametrize("hq,hkv", [(2, 2), (4, 2), (6, 2)], ids=["g1", "g2", "g3"])
def test_global_d512_group_sizes(hq, hkv):
    """Groups of 1, 2 and 3 query heads at d512: the O GEMM of the two-pass
    forward runs as 2-CTA head pairs for even groups, one CTA per head else."""
    _fixed_case(1, 300, 300, hq, hkv, 512, 0, seed=120 + hq)


def test_global_d512_rectangular_lower_right():
    _fixed_case(2, 70, 333, 8, 1, 512, 0, seed=7)


def test_local_d256_small_window_batch2():
    _fixed_case(2, 300, 300, 4, 2, 256, 100, seed=8)


def test_local_d256_vision_and_documents():
    s = 700
    rng = np.random.default_rng(3)
    vision = np.full((2, s), -1, dtype=np.int32)
    docs = np.zeros((2, s), dtype=np.int32)
    for b in range(2):
        for i, start in enumerate(sorted(rng.choice(np.arange(0, s - 90, 100), 4, replace=False))):
            vision[b, start:start + 90] = i
        docs[b, 420:] = 1
    vision[1, 650:690] = 0  # same id again later in the sequence (non-contiguous)
    _fixed_case(2, s, s, 4, 2, 256, 1024, seed=9, vision=vision, docs=docs)


def _packed_case(cu_q, cu_k, hq, hkv, d, window, seed, vision=None, docs=None):
    tq, tk = cu_q[-1], cu_k[-1]
    q, k, v = make_inputs((tq, hq, d), (tk, hkv, d), (tk, hkv, d), seed=seed, with_dout=False)
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    lq = np.diff(cu_q)
    lk = np.diff(cu_k)
    vis_t = None if vision is None else torch.tensor(vision, dtype=torch.int32, device="cuda")
    doc_t = None if docs is None else torch.tensor(docs, dtype=torch.int32, device="cuda")
    out, lse = ops.attn_fwd(q, k, v, window=window, cu_seqlens_q=cq, cu_seqlens_k=ck,
                            max_seqlen_q=int(lq.max()), max_seqlen_k=int(lk.max()),
                            vision_ids=vis_t, document_ids=doc_t)
    torch.cuda.synchronize()
    ref_o, ref_lse = oracle.attention_fwd_varlen(
        thd_np(q), thd_np(k), thd_np(v), cu_q, cu_k, sliding_window=window or None,
        allow_vision_bidirectional=window > 0,
        vision_block_ids=vision, document_ids=docs)
    assert rel_l2(out.float().cpu().numpy(), ref_o) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL


def test_local_d256_packed_with_empty_segments():
    _packed_case([0, 100, 100, 400, 1500], [0, 130, 200, 600, 1800], 4, 2, 256, 1024, seed=21)


def test_global_d512_packed():
    _packed_case([0, 5, 300, 301, 700], [0, 5, 300, 302, 900], 8, 1, 512, 0, seed=22)


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
    _packed_case(cu, cu, 4, 2, 256, 1024, seed=23, vision=vision, docs=docs)


def test_forward_is_bit_deterministic_on_side_stream():
    q, k, v = make_inputs((1, 777, 4, 256), (1, 777, 2, 256), (1, 777, 2, 256), seed=31,
                          with_dout=False)
    o1, l1 = ops.attn_fwd(q, k, v, window=1024)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o2, l2 = ops.attn_fwd(q, k, v, window=1024)
    s.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


@pytest.mark.parametrize("shape", [(1, 700, 8, 1, 0), (2, 300, 8, 1, 0)], ids=["b1", "b2"])
def test_global_two_pass_and_single_kernel_forward_agree_with_oracle(shape):
    b, s, hq, hkv, window = shape
    q, k, v = make_inputs((b, s, hq, 512), (b, s, hkv, 512), (b, s, hkv, 512), seed=91,
                          with_dout=False)
    ref_o, ref_lse = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k),
                                          bshd_to_bhsd_np(v))
    for algo in ("auto", "single"):
        out, lse = ops.attn_fwd(q, k, v, window=window, algorithm=algo)
        torch.cuda.synchronize()
        assert rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o)) <= REL_L2_TOL, algo
        assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL, algo


@pytest.mark.parametrize("algo", ["auto", "single"])
def test_global_rescales_when_the_running_max_jumps(algo):
    # Keys scaled by a growing ramp and queries aligned with their mean make the
    # row maxima climb by hundreds of log2 units across the key tiles, far past
    # the lazy-rescale threshold, so both forwards must rescale O repeatedly.
    s = 900
    q, k, v = make_inputs((1, s, 8, 512), (1, s, 1, 512), (1, s, 1, 512), seed=92,
                          with_dout=False)
    ramp = torch.linspace(0.1, 8.0, s, device="cuda").view(1, s, 1, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    q = (q.float() + 0.5 * k.float().mean(dim=1, keepdim=True).expand_as(q)).to(torch.bfloat16)
    ref_o, ref_lse = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k),
                                          bshd_to_bhsd_np(v))
    out, lse = ops.attn_fwd(q, k, v, window=0, algorithm=algo)
    torch.cuda.synchronize()
    assert rel_l2(out.float().cpu().numpy(), bhsd_to_bshd(ref_o)) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) <= LSE_ABS_TOL
