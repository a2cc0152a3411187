"""Opaque layer ops on the GPU at the Gemma-4 31B geometry: the whole local
and global layer forwards against an FP32 composition (FP32 projections,
norms and rotary; float64 attention oracle), the native kernels serving them
(fused preparation + attention), and the prepared BHSD ops against the
oracle.  Bars: output rel-L2 <= 2e-2 against the FP32 composition; the LSE
within 1e-3 of the oracle evaluated on the operands exactly as the op forms
them (BF16 projection, then the fused preparation)."""

import numpy as np
import pytest
import torch

import oracle
from parity_util import REL_L2_TOL, lse_abs_err, rel_l2

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib  # noqa: E402
from gemma4_fa4_kernels_b200 import layer_ops as L  # noqa: E402
from gemma4_fa4_kernels_b200.prep import prep_fwd  # noqa: E402

H = L.HIDDEN_SIZE


def _rms_norm(x, weight):
    xf = x.float()
    y = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + 1e-6, -0.5)
    return y if weight is None else y * weight.float()


def _rotary(x, cos, sin):
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos.unsqueeze(2) + rotated * sin.unsqueeze(2)


def _bhsd_np(x_bshd):
    return x_bshd.detach().double().cpu().numpy().transpose(0, 2, 1, 3)


def _setup(kind, s, seed):
    hq, hkv, d = L.LOCAL_GEOMETRY if kind == "local" else L.GLOBAL_GEOMETRY
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(1, s, H, generator=g).bfloat16().cuda()
    rope_angles = d // 2 if kind == "local" else d // 8  # global: 25% of frequencies rotated
    inv = 1.0 / (10_000.0 ** (torch.arange(0, 2 * rope_angles, 2, dtype=torch.float64) / d))
    inv = torch.cat((inv, torch.zeros(d // 2 - rope_angles, dtype=torch.float64)))
    ang = torch.arange(s, dtype=torch.float64)[:, None] * inv
    ang = torch.cat((ang, ang), dim=-1)[None]
    cos, sin = ang.cos().bfloat16().cuda(), ang.sin().bfloat16().cuda()

    def w(*shape):
        if len(shape) == 1:
            return (1.0 + 0.1 * torch.randn(*shape, generator=g)).bfloat16().cuda()
        return (torch.randn(*shape, generator=g) / shape[1] ** 0.5).bfloat16().cuda()

    weights = [w(hq * d, H), w(hkv * d, H)]
    if kind == "local":
        weights.append(w(hkv * d, H))
    weights += [w(H, hq * d), w(d), w(d)]
    pos = torch.arange(s, device="cuda").unsqueeze(0)
    packed = torch.zeros(1, s, dtype=torch.int64, device="cuda")
    return (hq, hkv, d), h, cos, sin, pos, packed, weights


@pytest.mark.parametrize("kind,s", [("local", 1), ("local", 1100), ("global", 300)])
@torch.no_grad()
def test_layer_forward_matches_the_fp32_composition(kind, s):
    (hq, hkv, d), h, cos, sin, pos, packed, weights = _setup(kind, s, seed=7 + s)
    if kind == "local":
        wq, wk, wv, wo, qn, kn = weights
    else:
        wq, wk, wo, qn, kn = weights
        wv = None
    n0 = _lib.launch_counts()
    fn = L.local_layer_fwd if kind == "local" else L.global_layer_fwd
    out, lse = fn(h, cos, sin, pos, packed, *weights)
    torch.cuda.synchronize()
    n1 = _lib.launch_counts()
    # Q, K and V(local) or Q and K/V(global, one launch) through the fused preparation
    assert n1["prep_fwd"] - n0["prep_fwd"] == (3 if kind == "local" else 2)
    assert sum(n1[k] - n0[k] for k in ("attn_fwd", "fwd_score", "decode", "decode_short")) >= 1
    assert out.shape == (1, s, H) and lse.shape == (1, hq, s)
    window = L.LOCAL_WINDOW if kind == "local" else None
    lin = torch.nn.functional.linear
    f = lambda t: t.float()  # noqa: E731
    # FP32 composition of the layer
    q = _rotary(_rms_norm(lin(f(h), f(wq)).view(1, s, hq, d), qn), f(cos), f(sin))
    z = lin(f(h), f(wk)).view(1, s, hkv, d)
    k = _rotary(_rms_norm(z, kn), f(cos), f(sin))
    v = _rms_norm(z if wv is None else lin(f(h), f(wv)).view(1, s, hkv, d), None)
    o, _ = oracle.attention_fwd(_bhsd_np(q), _bhsd_np(k), _bhsd_np(v), sliding_window=window,
                                allow_vision_bidirectional=kind == "local")
    ref_out = lin(torch.from_numpy(o).float().cuda().transpose(1, 2).reshape(1, s, hq * d), f(wo))
    assert rel_l2(out.float().cpu(), ref_out.cpu()) < 2e-2
    # the attention's LSE on the operands as the op forms them
    q_op, _ = prep_fwd(lin(h, wq).view(1, s, hq, d), qn, cos, sin, d)
    if kind == "local":
        k_op, _ = prep_fwd(lin(h, wk).view(1, s, hkv, d), kn, cos, sin, d)
        _, v_op = prep_fwd(lin(h, wv).view(1, s, hkv, d), None, None, None, 0, want_rot=False,
                           want_plain=True)
    else:
        k_op, v_op = prep_fwd(lin(h, wk).view(1, s, hkv, d), kn, cos, sin, d, want_plain=True)
    for name, got, ref in (("q", q_op, q), ("k", k_op, k), ("v", v_op, v)):
        assert rel_l2(got.float().cpu(), ref.cpu()) < REL_L2_TOL, name
    _, ref_lse = oracle.attention_fwd(_bhsd_np(q_op), _bhsd_np(k_op), _bhsd_np(v_op),
                                      sliding_window=window,
                                      allow_vision_bidirectional=kind == "local")
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) < 1e-3


@pytest.mark.parametrize("kind", ["local", "global"])
def test_prepared_ops_match_the_oracle(kind):
    hq, hkv, d = L.LOCAL_GEOMETRY if kind == "local" else L.GLOBAL_GEOMETRY
    s = 200
    g = torch.Generator().manual_seed(11)

    def unit(*shape):
        x = torch.randn(*shape, generator=g)
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).bfloat16().cuda()

    q, k, v = unit(1, hq, s, d), unit(1, hkv, s, d), unit(1, hkv, s, d)
    pos = torch.arange(s, device="cuda").unsqueeze(0)
    packed = torch.zeros(1, s, dtype=torch.int32, device="cuda")
    fn = L.local_fwd if kind == "local" else L.global_fwd
    out, lse = fn(q, k, v, pos, packed)
    torch.cuda.synchronize()
    assert out.shape == (1, s, hq, d) and lse.shape == (1, hq, s)
    to = lambda t: t.double().cpu().numpy()  # noqa: E731
    o, ref_lse = oracle.attention_fwd(to(q), to(k), to(v),
                                      sliding_window=L.LOCAL_WINDOW if kind == "local" else None,
                                      allow_vision_bidirectional=kind == "local")
    assert rel_l2(np.transpose(out.double().cpu().numpy(), (0, 2, 1, 3)), o) < REL_L2_TOL
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) < 1e-3
    bad = pos.clone()
    bad[0, -1] += 1
    from gemma4_fa4_kernels_b200 import UnsupportedB200Path

    with pytest.raises(UnsupportedB200Path, match="arange"):
        fn(q, k, v, bad, packed)
