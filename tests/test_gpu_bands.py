"""Banded materialised passes: the backward's P/dS tiles and the two-pass
forward's P tiles are processed band by band when the whole problem's scratch
exceeds the workspace.

Each case forces a workspace smaller than one band of the whole problem (the
``workspace_bytes`` override) and checks, through the C ABI:

* the result against the float64 oracle;
* against the same call with the whole-problem workspace: O, LSE and dQ are
  computed by the same CTA work in either plan and must be bit-identical; dK
  and dV of query bands are fp32 sums of per-band partials, within 1e-3;
* that several bands ran (launch counters), and which plan: bands of KV heads
  (every dV / dK complete, no conversion) or bands of query tiles (dV / dK
  summed in fp32 and converted once).

The gradient-accumulation mode (fp32 outputs that the call adds into) and the
causal shift used by ring context parallelism are checked here as well.
"""

import numpy as np
import pytest
import torch

from parity_util import (LSE_ABS_TOL, REL_L2_TOL, bshd_to_bhsd_np, make_inputs, rel_l2,
                         lse_abs_err, thd_np)

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import oracle  # noqa: E402
from gemma4_fa4_kernels_b200 import _lib, ops  # noqa: E402


def _counts():
    return _lib.launch_counts()


def _delta(before, after, name):
    return after[name] - before[name]


def _ws_sizes(q, k, v, out, lse, dout, window, **packed):
    import ctypes
    lib = _lib.load()
    a = ops._build_args(q, k, v, out, lse, window=window, vision_ids=None, document_ids=None,
                        cu_seqlens_q=packed.get("cu_seqlens_q"),
                        cu_seqlens_k=packed.get("cu_seqlens_k"),
                        max_seqlen_q=packed.get("max_seqlen_q"),
                        max_seqlen_k=packed.get("max_seqlen_k"))
    return (lib.g4_attn_bwd_workspace_bytes(ctypes.byref(a)),
            lib.g4_attn_bwd_min_workspace_bytes(ctypes.byref(a)),
            lib.g4_attn_fwd_workspace_bytes(ctypes.byref(a)),
            lib.g4_attn_fwd_min_workspace_bytes(ctypes.byref(a)))


def _np(t):
    return t.float().cpu().numpy()


def _check_grads(got, ref_np, to_np):
    for name, g, r in zip(("dq", "dk", "dv"), got, ref_np):
        err = rel_l2(to_np(g), r)
        assert err <= REL_L2_TOL, f"{name}: rel-L2 {err:.3e}"


@pytest.mark.parametrize("heads,frac,plan", [((8, 1), 0.6, "qtile"), ((16, 2), 0.55, "head")],
                         ids=["query_bands_gqa8", "kv_head_bands"])
def test_global_backward_in_bands(heads, frac, plan):
    hq, hkv = heads
    s, d = 1100, 512
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=5)
    out, lse = ops.attn_fwd(q, k, v)
    full, small, _, _ = _ws_sizes(q, k, v, out, lse, do, 0)
    ref = ops.attn_bwd(q, k, v, out, lse, do)
    before = _counts()
    got = ops.attn_bwd(q, k, v, out, lse, do, workspace_bytes=int(small + frac * (full - small)))
    after = _counts()
    torch.cuda.synchronize()
    assert _delta(before, after, "bwd_score") >= 2 * 2, "expected several bands (two passes each)"
    assert _delta(before, after, "bwd_dq") == 0 and _delta(before, after, "bwd_dkv") == 0
    casts = _delta(before, after, "cast_f32_bf16")
    assert casts == (2 if plan == "qtile" else 0)
    assert torch.equal(got[0], ref[0]), "dQ must not depend on the band plan"
    for g, r in zip(got[1:], ref[1:]):
        assert rel_l2(_np(g), _np(r)) <= 1e-3
    rq, rk, rv = oracle.attention_bwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
                                      bshd_to_bhsd_np(do))
    _check_grads(got, (rq, rk, rv), bshd_to_bhsd_np)


def test_global_two_pass_forward_in_bands():
    hq, hkv, s, d = 8, 1, 1300, 512
    q, k, v = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=6, with_dout=False)
    o_ref, l_ref = ops.attn_fwd(q, k, v)
    _, _, full, small = _ws_sizes(q, k, v, o_ref, l_ref, None, 0)
    before = _counts()
    o, l = ops.attn_fwd(q, k, v, workspace_bytes=int(small + 0.3 * (full - small)))
    after = _counts()
    torch.cuda.synchronize()
    assert _delta(before, after, "fwd_score") >= 2
    assert _delta(before, after, "attn_fwd") == 0
    assert torch.equal(o, o_ref) and torch.equal(l, l_ref)
    ro, rl = oracle.attention_fwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v))
    assert rel_l2(bshd_to_bhsd_np(o), ro) <= REL_L2_TOL
    assert lse_abs_err(l.cpu().numpy(), rl) <= LSE_ABS_TOL


def test_local_backward_in_bands():
    hq, hkv, s, d, w = 4, 2, 2300, 256, 1024
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=7)
    out, lse = ops.attn_fwd(q, k, v, window=w)
    full, small, _, _ = _ws_sizes(q, k, v, out, lse, do, w)
    ref = ops.attn_bwd(q, k, v, out, lse, do, window=w)
    before = _counts()
    got = ops.attn_bwd(q, k, v, out, lse, do, window=w,
                       workspace_bytes=int(small + 0.45 * (full - small)))
    after = _counts()
    torch.cuda.synchronize()
    assert _delta(before, after, "bwd_score") >= 2
    assert torch.equal(got[0], ref[0])
    for g, r in zip(got[1:], ref[1:]):
        assert rel_l2(_np(g), _np(r)) <= 1e-3
    rq, rk, rv = oracle.attention_bwd(bshd_to_bhsd_np(q), bshd_to_bhsd_np(k), bshd_to_bhsd_np(v),
                                      bshd_to_bhsd_np(do), sliding_window=w)
    _check_grads(got, (rq, rk, rv), bshd_to_bhsd_np)


def test_packed_global_in_bands():
    """Packed segments: the band plan reads cu_seqlens back to the host."""
    lens = [300, 0, 700, 129, 1]
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    t, hq, hkv, d = int(sum(lens)), 8, 1, 512
    q, k, v, do = make_inputs((t, hq, d), (t, hkv, d), (t, hkv, d), seed=8)
    kw = dict(cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(lens), max_seqlen_k=max(lens))
    o_ref, l_ref = ops.attn_fwd(q, k, v, **kw)
    full, small, ffull, fsmall = _ws_sizes(q, k, v, o_ref, l_ref, do, 0, **kw)
    ref = ops.attn_bwd(q, k, v, o_ref, l_ref, do, **kw)
    before = _counts()
    o, l = ops.attn_fwd(q, k, v, workspace_bytes=int(fsmall + 0.25 * (ffull - fsmall)), **kw)
    got = ops.attn_bwd(q, k, v, o_ref, l_ref, do, workspace_bytes=int(small + 0.25 * (full - small)),
                       **kw)
    after = _counts()
    torch.cuda.synchronize()
    assert _delta(before, after, "fwd_score") >= 2 and _delta(before, after, "bwd_score") >= 4
    assert torch.equal(o, o_ref) and torch.equal(l, l_ref)
    assert torch.equal(got[0], ref[0])
    for g, r in zip(got[1:], ref[1:]):
        assert rel_l2(_np(g), _np(r)) <= 1e-3
    cu_np = cu.cpu().numpy()
    _, _, rq, rk, rv = oracle.attention_fwd_bwd_varlen(thd_np(q), thd_np(k), thd_np(v),
                                                       thd_np(do), cu_np, cu_np)
    _check_grads(got, (rq, rk, rv), thd_np)


def test_gradient_accumulation_adds_into_fp32():
    hq, hkv, s, d = 8, 1, 700, 512
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=9)
    out, lse = ops.attn_fwd(q, k, v)
    ref = ops.attn_bwd(q, k, v, out, lse, do)
    acc = [torch.zeros(t.shape, dtype=torch.float32, device="cuda") for t in (q, k, v)]
    full, small, _, _ = _ws_sizes(q, k, v, out, lse, do, 0)
    for ws in (None, int(small + 0.6 * (full - small))):  # one band, then query bands
        ops.attn_bwd(q, k, v, out, lse, do, dq=acc[0], dk=acc[1], dv=acc[2], accumulate=True,
                     workspace_bytes=ws)
    torch.cuda.synchronize()
    for a, r in zip(acc, ref):
        assert rel_l2(a.cpu().numpy(), 2 * _np(r)) <= 2e-3


@pytest.mark.parametrize("sq,sk,shift", [(700, 900, 0), (700, 900, 64), (700, 900, 700),
                                         (900, 500, 900), (1200, 600, 1200)],
                         ids=["none", "partial", "all_keys", "more_queries_than_keys",
                              "ring_early_chunk"])
def test_causal_shift(sq, sk, shift):
    hq, hkv, d = 8, 1, 512
    q, k, v, do = make_inputs((1, sq, hq, d), (1, sk, hkv, d), (1, sk, hkv, d), seed=10)
    out, lse = ops.attn_fwd(q, k, v, causal_shift=shift)
    dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, do, causal_shift=shift)
    torch.cuda.synchronize()
    qn, kn, vn, don = (bshd_to_bhsd_np(t) for t in (q, k, v, do))
    # The oracle keeps queries inside the key stream, so the shift is expressed
    # as `shift` padded keys after the real ones (masked by key padding).
    pad = lambda x: np.concatenate([x, np.zeros(x.shape[:2] + (shift, x.shape[3]))], axis=2)  # noqa
    keep = np.concatenate([np.ones((1, sk), bool), np.zeros((1, shift), bool)], axis=1)
    kw = dict(q_start=sk - sq + shift, key_padding_mask=keep)
    ro, rl = oracle.attention_fwd(qn, pad(kn), pad(vn), **kw)
    rq, rk, rv = oracle.attention_bwd(qn, pad(kn), pad(vn), don, **kw)
    rk, rv = rk[:, :, :sk], rv[:, :, :sk]
    assert rel_l2(bshd_to_bhsd_np(out), ro) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), rl) <= LSE_ABS_TOL
    _check_grads((dq, dk, dv), (rq, rk, rv), bshd_to_bhsd_np)



def test_local_many_short_segments():
    """Packed local d256 attention over many short segments (1 to 300 tokens):
    the persistent forward walks hundreds of one-to-three-tile items, so the
    look-ahead across items (the next item's Q and first S before the current
    item's last P V) and the epilogue warps' hand-over run at almost every
    tile.  Every segment is checked against the float64 oracle."""
    rng = np.random.default_rng(12)
    lens = [int(x) for x in rng.integers(1, 301, size=40)]
    lens[3] = 128
    lens[7] = 129
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device="cuda")
    t, hq, hkv, d, w = int(sum(lens)), 4, 2, 256, 256
    q, k, v, do = make_inputs((t, hq, d), (t, hkv, d), (t, hkv, d), seed=12)
    kw = dict(cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(lens), max_seqlen_k=max(lens),
              window=w)
    out, lse = ops.attn_fwd(q, k, v, **kw)
    dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, do, **kw)
    torch.cuda.synchronize()
    cu_np = cu.cpu().numpy()
    ro, rl, rq, rk, rv = oracle.attention_fwd_bwd_varlen(thd_np(q), thd_np(k), thd_np(v),
                                                         thd_np(do), cu_np, cu_np,
                                                         sliding_window=w)
    assert rel_l2(thd_np(out), ro) <= REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), rl) <= LSE_ABS_TOL
    _check_grads((dq, dk, dv), (rq, rk, rv), thd_np)
