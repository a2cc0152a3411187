"""GPU parity of the fused Q/K/V preparation (``g4_prep_fwd`` / ``g4_prep_bwd``)
against the float64 oracle, on the reference test's geometries and on Gemma-4
layer shapes (global shared source d512, local d256, packed rows, strided
projection views).  Bar: rel-L2 <= 1e-2 against the oracle on the same BF16
inputs, and no worse than twice the error of the BF16 eager composition the
reference layer ops run (h100_torch_ops.py:302-326)."""

import numpy as np
import pytest
import torch

from oracle import prep as oprep
from parity_util import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib  # noqa: E402
from gemma4_fa4_kernels_b200 import prep  # noqa: E402


def _np(t):
    return None if t is None else t.detach().double().cpu().numpy()


def _eager(x, w, cos, sin, rd, head_axis, drot=None, dplain=None):
    """The reference layer ops' BF16 order: FP32 norm cast back to BF16, then
    the rotary products in BF16 (h100_torch_ops.py:302-326), under autograd."""
    x = x.detach().clone().requires_grad_(True)
    wp = None if w is None else w.detach().clone().requires_grad_(True)
    xf = x.float()
    n = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + 1e-6, -0.5)
    plain = n.type_as(x)
    nw = (n * wp.float()).type_as(x) if wp is not None else plain
    if rd:
        c, s = cos.unsqueeze(head_axis), sin.unsqueeze(head_axis)
        r = nw[..., :rd]
        rot_half = torch.cat((-r[..., rd // 2:], r[..., : rd // 2]), dim=-1)
        rot = torch.cat((r * c + rot_half * s, nw[..., rd:]), dim=-1)
    else:
        rot = nw
    outs, grads = [], []
    if drot is not None:
        outs.append(rot)
        grads.append(drot)
    if dplain is not None:
        outs.append(plain)
        grads.append(dplain)
    if outs:
        torch.autograd.backward(outs, grads)
    return rot.detach(), plain.detach(), x.grad, None if wp is None else wp.grad


def _check(name, got, ref, eager=None, tol=REL_L2_TOL):
    e = rel_l2(got, ref)
    assert e <= tol, f"{name}: rel-L2 {e:.3e} > {tol}"
    if eager is not None:
        ee = rel_l2(eager, ref)
        assert e <= 2 * ee + 1e-6, f"{name}: {e:.3e} worse than 2x eager {ee:.3e}"


def _tables_np(cos, sin, head_axis):
    return np.expand_dims(_np(cos), head_axis), np.expand_dims(_np(sin), head_axis)


def _run_case(x, w, cos, sin, rd, layout, *, seed, plain=True):
    head_axis = {"bshd": 2, "bhsd": 1, "thd": 1}[layout]
    g = torch.Generator().manual_seed(seed)
    drot = torch.randn(x.shape, generator=g).to(torch.bfloat16).cuda()
    dplain = torch.randn(x.shape, generator=g).to(torch.bfloat16).cuda() if plain else None
    n0 = _lib.launch_counts()
    rot, pl = prep.prep_fwd(x, w, cos, sin, rd, layout=layout, want_plain=plain)
    dx, dw = prep.prep_bwd(x, w, cos, sin, rd, drot, dplain, layout=layout)
    torch.cuda.synchronize()
    n1 = _lib.launch_counts()
    assert n1["prep_fwd"] == n0["prep_fwd"] + 1 and n1["prep_bwd"] == n0["prep_bwd"] + 1
    c_np, s_np = _tables_np(cos, sin, head_axis) if rd else (None, None)
    xn, wn = _np(x), _np(w)
    ref_rot = oprep.apply_partial_rotary(oprep.rms_norm(xn, wn), c_np, s_np, rd)
    ref_plain = oprep.rms_norm(xn)
    ref_dx, ref_dw = oprep.prepare_bwd(xn, wn, c_np, s_np, rd, _np(drot), _np(dplain))
    if layout == "thd":  # the eager yardstick broadcasts (T, R) tables over heads
        e_rot, e_plain, e_dx, e_dw = _eager(x, w, cos, sin, rd, 1, drot, dplain)
    else:
        e_rot, e_plain, e_dx, e_dw = _eager(x, w, cos, sin, rd, head_axis, drot, dplain)
    _check("rot", _np(rot), ref_rot, _np(e_rot))
    if plain:
        _check("plain", _np(pl), ref_plain, _np(e_plain))
    _check("dx", _np(dx), ref_dx, _np(e_dx))
    if w is not None:
        _check("dweight", _np(dw), ref_dw, _np(e_dw))
    return rot, pl, dx, dw


def test_reference_test_geometries():
    # The shapes of the reference's own preparation test
    # (tests/test_reference.py:381-407): a (1, 2, 3, 512) source in the helper's
    # (B, H, S, D) layout, 128 rotated features, weight linspace(0.75, 1.25);
    # and the layer ops' order on a (1, 3, 2, 256) operand with full tables.
    # The oracle these are checked against is pinned to the reference's
    # float64 outputs by the CPU golden tests.
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 2, 3, 512, generator=g).to(torch.bfloat16).cuda()
    w = torch.linspace(0.75, 1.25, 512).to(torch.bfloat16).cuda()
    ang = torch.linspace(0.01, 0.91, 3 * 128, dtype=torch.float64).reshape(1, 3, 128)
    _run_case(x, w, ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda(),
              128, "bhsd", seed=1)
    x = torch.randn(1, 3, 2, 256, generator=g).to(torch.bfloat16).cuda()
    w = (1.0 + 0.3 * torch.randn(256, generator=g)).to(torch.bfloat16).cuda()
    ang = torch.rand(1, 3, 128, generator=g, dtype=torch.float64) * 6.0
    ang = torch.cat((ang, ang), dim=-1)
    _run_case(x, w, ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda(),
              256, "bshd", seed=2)


def _hf_tables(s, d, rope_angles, base, seed, batch=1):
    """Full-width Gemma tables: ``rope_angles`` rotated frequency pairs, the
    other (d/2 - rope_angles) frequencies zero (cos 1, sin 0), positions
    0..s-1 plus a seeded offset."""
    g = torch.Generator().manual_seed(seed)
    inv = 1.0 / (base ** (torch.arange(0, 2 * rope_angles, 2, dtype=torch.float64) / d))
    inv = torch.cat((inv, torch.zeros(d // 2 - rope_angles, dtype=torch.float64)))
    pos = torch.arange(s, dtype=torch.float64)[None] + torch.randint(0, 5000, (batch, 1), generator=g)
    ang = pos[..., None] * inv
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()


def _source(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).cuda()


def _norm_weight(d, seed):
    g = torch.Generator().manual_seed(seed)
    return (1.0 + 0.2 * torch.randn(d, generator=g)).to(torch.bfloat16).cuda()


def test_global_shared_source_d512_proportional_tables():
    # global layer: Z (B, S, 4, 512), 25% of the frequencies rotated
    x = _source((2, 300, 4, 512), 11, scale=3.0)
    cos, sin = _hf_tables(300, 512, 64, 1_000_000.0, 12, batch=2)
    _run_case(x, _norm_weight(512, 13), cos, sin, 512, "bshd", seed=14)


def test_global_partial_subspace_bhsd_like_the_reference_helper():
    x = _source((1, 4, 257, 512), 21)
    g = torch.Generator().manual_seed(22)
    ang = torch.rand(1, 257, 128, generator=g, dtype=torch.float64) * 6.0
    _run_case(x, _norm_weight(512, 23), ang.cos().to(torch.bfloat16).cuda(),
              ang.sin().to(torch.bfloat16).cuda(), 128, "bhsd", seed=24)


def test_local_query_d256_from_a_strided_projection_view():
    # Q as a view into a wider projection buffer: head stride 512, token stride 32*512
    big = _source((1, 129, 32, 512), 31)
    x = big[..., 128:384]
    assert not x.is_contiguous()
    cos, sin = _hf_tables(129, 256, 128, 10_000.0, 32)
    _run_case(x, _norm_weight(256, 33), cos, sin, 256, "bshd", seed=34, plain=False)


def test_packed_rows_and_no_rotation():
    x = _source((1000, 16, 256), 41)
    g = torch.Generator().manual_seed(42)
    ang = torch.rand(1000, 64, generator=g, dtype=torch.float64) * 6.0
    _run_case(x, _norm_weight(256, 43), ang.cos().to(torch.bfloat16).cuda(),
              ang.sin().to(torch.bfloat16).cuda(), 64, "thd", seed=44)
    _run_case(_source((3, 7, 2, 512), 45), _norm_weight(512, 46), None, None, 0, "bshd", seed=47)


def test_odd_row_counts_d256():
    # d256 rows go two per warp step: odd totals leave a half-empty last step
    for shape, seed in (((1, 7, 3, 256), 81), ((1, 1, 1, 256), 82), ((2, 333, 3, 256), 83)):
        cos, sin = _hf_tables(shape[1], 256, 128, 10_000.0, seed, batch=shape[0])
        _run_case(_source(shape, seed), _norm_weight(256, seed), cos, sin, 256, "bshd", seed=seed)


def test_value_only_and_no_weight():
    x = _source((1, 70, 16, 256), 51, scale=0.01)  # tiny magnitudes: eps matters
    g = torch.Generator().manual_seed(52)
    dv = torch.randn(x.shape, generator=g).to(torch.bfloat16).cuda()
    _, v = prep.prep_fwd(x, None, None, None, 0, want_rot=False, want_plain=True)
    dx, dw = prep.prep_bwd(x, None, None, None, 0, None, dv)
    assert dw is None
    ref_dx, _ = oprep.prepare_bwd(_np(x), None, None, None, 0, None, _np(dv))
    _, e_plain, e_dx, _ = _eager(x, None, None, None, 0, 2, None, dv)
    _check("plain", _np(v), oprep.rms_norm(_np(x)), _np(e_plain))
    _check("dx", _np(dx), ref_dx, _np(e_dx))


def test_autograd_surface_and_determinism():
    x = _source((1, 2, 64, 512), 61).requires_grad_(True)
    w = _norm_weight(512, 62).requires_grad_(True)
    g = torch.Generator().manual_seed(63)
    ang = torch.rand(1, 64, 128, generator=g, dtype=torch.float64) * 6.0
    cos, sin = ang.cos().to(torch.bfloat16).cuda(), ang.sin().to(torch.bfloat16).cuda()
    k, v = prep.prepare_global_kv_from_projection_source(x, k_norm_weight=w, cos=cos, sin=sin)
    assert k.data_ptr() != v.data_ptr()
    gk = torch.randn(k.shape, generator=g).to(torch.bfloat16).cuda()
    gv = torch.randn(v.shape, generator=g).to(torch.bfloat16).cuda()
    torch.autograd.backward((k, v), (gk, gv))
    dx1, dw1 = x.grad.clone(), w.grad.clone()
    x.grad, w.grad = None, None
    k, v = prep.prepare_global_kv_from_projection_source(x, k_norm_weight=w, cos=cos, sin=sin)
    torch.autograd.backward((k, v), (gk, gv))
    assert torch.equal(dx1, x.grad) and torch.equal(dw1, w.grad)
    c_np, s_np = _tables_np(cos, sin, 1)
    ref_dx, ref_dw = oprep.prepare_bwd(_np(x), _np(w), c_np, s_np, 128, _np(gk), _np(gv))
    _check("dx", _np(dx1), ref_dx)
    _check("dweight", _np(dw1), ref_dw)
    # K only (no gradient reaches V): the V-side adjoint drops out
    x.grad, w.grad = None, None
    k, _ = prep.prepare_global_kv_from_projection_source(x, k_norm_weight=w, cos=cos, sin=sin)
    k.backward(gk)
    ref_dx, _ = oprep.prepare_bwd(_np(x), _np(w), c_np, s_np, 128, _np(gk), None)
    _check("dx (K only)", _np(x.grad), ref_dx)


def test_empty_rows():
    x = torch.empty(1, 0, 4, 512, dtype=torch.bfloat16, device="cuda")
    w = _norm_weight(512, 71)
    rot, pl = prep.prep_fwd(x, w, None, None, 0, want_plain=True)
    dx, dw = prep.prep_bwd(x, w, None, None, 0, torch.empty_like(x), None)
    torch.cuda.synchronize()
    assert rot.numel() == 0 and pl.numel() == 0 and dx.numel() == 0
    assert torch.count_nonzero(dw) == 0
