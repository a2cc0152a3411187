"""Pin the numpy oracle to golden vectors recorded from the reference project.

The fixtures in ``tests/golden`` were produced by ``tests/golden/make_golden.py``
importing the reference ``gemma4_fa4`` package (float64 torch autograd).
These CPU tests prove the oracle reproduces them before any CUDA result is
compared against the oracle.
"""

import glob
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _meta(z):
    return json.loads(str(z["meta"]))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_fixed_attention_matches_reference_golden(path):
    z = np.load(path)
    meta = _meta(z)
    window = None if meta["window"] < 0 else meta["window"]
    kw = dict(sliding_window=window, allow_vision_bidirectional=bool(meta["bidir"]),
              vision_block_ids=z["vision"] if "vision" in z else None,
              document_ids=z["docs"] if "docs" in z else None,
              key_padding_mask=z["padding"] if "padding" in z else None)
    out, lse = oracle.attention_fwd(z["q"], z["k"], z["v"], **kw)
    np.testing.assert_allclose(out, z["out"], rtol=1e-12, atol=1e-12)
    np.testing.assert_array_equal(np.isneginf(lse), np.isneginf(z["lse"]))
    fin = np.isfinite(z["lse"])
    np.testing.assert_allclose(lse[fin], z["lse"][fin], rtol=1e-6, atol=1e-6)
    dq, dk, dv = oracle.attention_bwd(z["q"], z["k"], z["v"], z["dout"],
                                      dlse=z["dlse"] if "dlse" in z else None, **kw)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, z[name], rtol=1e-10, atol=1e-10, err_msg=name)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "varlen_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_varlen_attention_matches_reference_golden(path):
    z = np.load(path)
    meta = _meta(z)
    window = None if meta["window"] < 0 else meta["window"]
    out, lse, dq, dk, dv = oracle.attention_fwd_bwd_varlen(
        z["q"], z["k"], z["v"], z["dout"], z["cu_q"], z["cu_k"], sliding_window=window,
        vision_block_ids=z["vision"] if "vision" in z else None,
        document_ids=z["docs"] if "docs" in z else None,
        allow_vision_bidirectional=bool(meta["bidir"]))
    np.testing.assert_allclose(out, z["out"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(lse, z["lse"], rtol=1e-6, atol=1e-6)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        np.testing.assert_allclose(got, z[name], rtol=1e-10, atol=1e-10, err_msg=name)


def test_masks_match_reference_golden_bit_exact():
    with open(os.path.join(GOLD, "masks.json")) as f:
        cases = json.load(f)
    assert len(cases) >= 20
    for name, c in cases.items():
        m = oracle.gemma4_attention_mask(
            batch_size=c["b"], q_len=c["q_len"], kv_len=c["kv_len"], sliding_window=c["window"],
            vision_block_ids=None if c["vision"] is None else np.asarray(c["vision"]),
            document_ids=None if c["docs"] is None else np.asarray(c["docs"]),
            key_padding_mask=None if c["padding"] is None else np.asarray(c["padding"]),
            allow_vision_bidirectional=c["bidir"])
        np.testing.assert_array_equal(m.astype(np.uint8), np.asarray(c["mask"], np.uint8).reshape(c["shape"]),
                                      err_msg=name)


def test_sparse_schedules_match_reference_golden_exactly():
    with open(os.path.join(GOLD, "schedules.json")) as f:
        cases = json.load(f)
    assert cases["upper_bound_262144"] == 94_027_776
    assert oracle.local_sparse_storage_upper_bound(262144, 262144) == 94_027_776
    n = 0
    for name, c in cases.items():
        if not name.startswith("case"):
            continue
        s = oracle.build_local_sparse_schedule(
            c["vision"], c["docs"], q_length=c["q_length"], k_length=c["k_length"],
            sliding_window=c["window"], forward_block_size=tuple(c["forward_block_size"]),
            backward_block_size=tuple(c["backward_block_size"]))
        assert [list(r) for r in s["forward"]] == c["forward"], name
        assert [list(r) for r in s["backward"]] == c["backward"], name
        assert s["forward_storage_bytes"] == c["forward_storage_bytes"], name
        assert s["backward_storage_bytes"] == c["backward_storage_bytes"], name
        n += 1
    assert n >= 30


def test_flops_match_reference_golden():
    with open(os.path.join(GOLD, "flops.json")) as f:
        cases = json.load(f)
    for key, value in cases.items():
        kind, s, mode = key.split("_", 2)
        if kind == "local":
            got = oracle.attention_flops(num_q_heads=32, head_dim_qk=256, head_dim_v=256, batch=1,
                                         seqlen=int(s), sliding_window=1024, mode=mode)
        else:
            got = oracle.attention_flops(num_q_heads=32, head_dim_qk=512, head_dim_v=512, batch=1,
                                         seqlen=int(s), sliding_window=None, mode=mode)
        assert got == value, key


# ---- known-answer tests restated from the reference's own test-suite -------------------

def test_kat_lower_right_vision_truth_table():
    # test_reference.py:307-328 -> O = 1.5
    q = np.zeros((3, 1, 1))
    k = np.zeros((5, 1, 1))
    v = np.arange(5, dtype=np.float64).reshape(5, 1, 1)
    out, _ = oracle.attention_fwd_varlen(q, k, v, [0, 3], [0, 5], sliding_window=1024,
                                         vision_block_ids=np.array([-1, -1, 7, 7, 8]),
                                         allow_vision_bidirectional=True)
    assert out[0, 0, 0] == 1.5


def test_kat_strict_w1024_lower_edge():
    # test_reference.py:331-356 -> O = 1/1024
    q = np.zeros((1, 1, 1))
    k = np.zeros((1025, 1, 1))
    v = np.zeros_like(k)
    v[0] = 100
    v[1] = 1
    out, _ = oracle.attention_fwd_varlen(q, k, v, [0, 1], [0, 1025], sliding_window=1024,
                                         vision_block_ids=np.zeros(1025, np.int64),
                                         allow_vision_bidirectional=True)
    assert math.isclose(out[0, 0, 0], 1.0 / 1024.0, rel_tol=1e-12)


def test_kat_window_one_returns_v():
    # test_reference.py:64-69
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 4, 8)) for _ in range(3))
    out, _ = oracle.attention_fwd(q, k, v, sliding_window=1)
    np.testing.assert_allclose(out, v, atol=1e-12)


def test_kat_analytic_long_context():
    # The reference's long-context analytic oracle (Q=0, K=1, V=0.25): every
    # allowed key has equal weight, so O = 0.25 and LSE = log(#keys).
    s = 300
    q = np.zeros((1, 1, s, 4))
    k = np.ones((1, 1, s, 4))
    v = np.full((1, 1, s, 4), 0.25)
    out, lse = oracle.attention_fwd(q, k, v)
    np.testing.assert_allclose(out, 0.25, atol=1e-15)
    np.testing.assert_allclose(lse[0, 0], np.log(np.arange(1, s + 1)), rtol=1e-6)


def test_mask_aware_pairs_text_matches_closed_form():
    for s, w in ((2048, 1024), (4096, None), (100, 1024), (1025, 1024)):
        assert oracle.mask_aware_pairs(q_len=s, kv_len=s, sliding_window=w) == \
            oracle.valid_pair_count(s, w)
    assert oracle.valid_pair_count(2048, 1024) == 1_573_376
    assert oracle.valid_pair_count(4096, None) == 8_390_656


@pytest.mark.parametrize("name,layout", [("global_kv_partial", "bhsd"), ("layer_full_d256", "bshd")])
def test_prep_oracle_matches_reference_golden(name, layout):
    # The reference computes the RMS statistics through ``x.float()`` even for
    # float64 inputs (reference.py:277, h100_torch_ops.py:308), so its float64
    # fixtures carry float32 rounding of the norm: agreement is to ~1e-6.
    from oracle import prep

    z = np.load(os.path.join(GOLD, f"prep_{name}.npz"))
    rd = int(z["rotary_dim"])
    axis = 1 if layout == "bhsd" else 2  # where the head axis sits in x
    cos, sin = np.expand_dims(z["cos"], axis), np.expand_dims(z["sin"], axis)
    rot = prep.apply_partial_rotary(prep.rms_norm(z["x"], z["weight"]), cos, sin, rd)
    np.testing.assert_allclose(rot, z["rot"], rtol=0, atol=5e-6)
    np.testing.assert_allclose(prep.rms_norm(z["x"]), z["plain"], rtol=0, atol=5e-6)
    dx, dw = prep.prepare_bwd(z["x"], z["weight"], cos, sin, rd, z["g_rot"], z["g_plain"])
    np.testing.assert_allclose(dx, z["dx"], rtol=0, atol=5e-6)
    np.testing.assert_allclose(dw, z["dweight"], rtol=1e-5, atol=5e-6)
    if name == "global_kv_partial":
        k, v = prep.prepare_global_kv(z["x"], z["weight"], cos, sin, 0.25)
        np.testing.assert_allclose(k, z["rot"], rtol=0, atol=5e-6)
        np.testing.assert_allclose(v, z["plain"], rtol=0, atol=5e-6)


def test_prep_rotary_adjoint_is_the_transpose():
    from oracle import prep

    rng = np.random.default_rng(5)
    for rd in (0, 8, 16, 32):
        x, g = rng.standard_normal((3, 32)), rng.standard_normal((3, 32))
        ang = rng.uniform(0, 6, size=(3, rd))
        c, s = np.cos(ang), np.sin(ang)
        lhs = np.sum(prep.apply_partial_rotary(x, c, s, rd) * g)
        rhs = np.sum(x * prep.rotary_adjoint(g, c, s, rd))
        assert abs(lhs - rhs) < 1e-12


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p))
def test_torch_cpu_baseline_matches_reference_golden(path):
    """The torch restatement timed as bench.py's CPU baseline reproduces the
    reference's outputs and autograd gradients (float64, and float32 upcast
    within float32 rounding)."""
    import torch

    from oracle.attention_torch import reference_attention_torch

    z = np.load(path)
    if "padding" in z:
        pytest.skip("key padding is not part of the benchmarked configurations")
    meta = _meta(z)
    window = None if meta["window"] < 0 else meta["window"]
    kw = dict(sliding_window=window, allow_vision_bidirectional=bool(meta["bidir"]),
              vision_block_ids=z["vision"] if "vision" in z else None,
              document_ids=z["docs"] if "docs" in z else None)
    for upcast, tol in ((torch.float64, 1e-10), (torch.float32, 2e-4)):
        q, k, v = (torch.from_numpy(z[n]).requires_grad_(True) for n in ("q", "k", "v"))
        out, lse = reference_attention_torch(q, k, v, upcast=upcast, **kw)
        loss = (out * torch.from_numpy(z["dout"])).sum()
        if "dlse" in z:
            dl = torch.from_numpy(z["dlse"])
            loss = loss + torch.where(torch.isfinite(lse), lse.double() * dl, torch.zeros_like(dl)).sum()
        loss.backward()
        np.testing.assert_allclose(out.detach().numpy(), z["out"], rtol=tol, atol=tol)
        for t, name in ((q, "dq"), (k, "dk"), (v, "dv")):
            np.testing.assert_allclose(t.grad.numpy(), z[name], rtol=tol * 10, atol=tol * 10,
                                       err_msg=name)
