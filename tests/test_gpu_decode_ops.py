"""Static-cache decode ops on the GPU at the Gemma-4 31B geometry: cache
mutation (new slot written, other slots untouched, the local window rolled),
``cache_length`` bookkeeping, the decode kernel serving the attention, and the
outputs against an FP32 composition of the same layer with the float64
attention oracle."""

import pytest
import torch

import oracle
from parity_util import lse_abs_err, rel_l2

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib  # noqa: E402
from gemma4_fa4_kernels_b200 import decode_ops as d  # noqa: E402
from gemma4_fa4_kernels_b200.prep import prep_fwd  # noqa: E402

H = d.HIDDEN_SIZE


def _rms_norm(x, weight):
    """Gemma RMS norm in FP32 (eps 1e-6), optional scale (h100_torch_ops.py:302-313)."""
    xf = x.float()
    y = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + 1e-6, -0.5)
    return y if weight is None else y * weight.float()


def _rotary(x, cos, sin):
    """x * cos + rotate_half(x) * sin on (B, S, H, D) with (B, S, D) tables."""
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos.unsqueeze(2) + rotated * sin.unsqueeze(2)


def _rms_unit(x):
    return x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)


def _weights(g, shapes):
    out = []
    for s in shapes:
        if len(s) == 1:
            out.append((1.0 + 0.1 * torch.randn(*s, generator=g)).bfloat16().cuda())
        else:
            out.append((torch.randn(*s, generator=g) / s[1] ** 0.5).bfloat16().cuda())
    return out


def _rope(g, dim):
    ang = torch.rand(1, 1, dim // 2, generator=g) * 6.28
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos().bfloat16().cuda(), ang.sin().bfloat16().cuda()


def _ref_layer(h, cos, sin, wq, wk, wv, wo, qn, kn, cache_k, cache_v, active, hq, hkv, dim,
               window):
    """FP32 composition: projections, norms and rotary in FP32 from the BF16
    operands; attention in float64 over the op's BF16 cache contents.  Also
    returns the float64 LSE for the query exactly as the op forms it (BF16
    projection, then the fused preparation kernel), which isolates the
    attention kernel: with d512 scores near 80, BF16 rounding of Q alone moves
    the LSE by ~0.1."""
    f = lambda t: t.float()  # noqa: E731
    lin = torch.nn.functional.linear
    q = _rotary(_rms_norm(lin(f(h), f(wq)).view(1, 1, hq, dim), qn), f(cos), f(sin))
    z = lin(f(h), f(wk)).view(1, 1, hkv, dim)
    k_new = _rotary(_rms_norm(z, kn), f(cos), f(sin))
    v_new = _rms_norm(z if wv is None else lin(f(h), f(wv)).view(1, 1, hkv, dim), None)
    kk = cache_k[:, :, :active].double().cpu().numpy()
    vv = cache_v[:, :, :active].double().cpu().numpy()
    o, _ = oracle.attention_fwd(q.transpose(1, 2).double().cpu().numpy(), kk, vv,
                                sliding_window=window)
    out = lin(torch.from_numpy(o).float().cuda().transpose(1, 2).reshape(1, 1, hq * dim), f(wo))
    q_bf, _ = prep_fwd(lin(h, wq).view(1, 1, hq, dim), qn, cos, sin, dim)
    _, lse_bf = oracle.attention_fwd(q_bf.transpose(1, 2).double().cpu().numpy(), kk, vv,
                                     sliding_window=window)
    return out, lse_bf, k_new, v_new


@torch.no_grad()
def test_global_decode_step_writes_one_slot_and_attends_over_the_prefix():
    g = torch.Generator().manual_seed(1)
    cap, length = 3000, 2500
    h = torch.randn(1, 1, H, generator=g).bfloat16().cuda()
    cos, sin = _rope(g, 512)
    wq, wk, wo, qn, kn = _weights(g, [(32 * 512, H), (4 * 512, H), (H, 32 * 512), (512,), (512,)])
    cache_k = torch.zeros(1, 4, cap, 512, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    cache_k[:, :, :length] = _rms_unit(torch.randn(1, 4, length, 512, generator=g)).bfloat16().cuda()
    cache_v[:, :, :length] = _rms_unit(torch.randn(1, 4, length, 512, generator=g)).bfloat16().cuda()
    before_k, before_v = cache_k.clone(), cache_v.clone()
    cache_length = torch.tensor(length, dtype=torch.int64, device="cuda")
    pos = torch.full((1, 1), length, dtype=torch.int64, device="cuda")
    n0 = _lib.launch_counts()["decode"]
    out, lse = d.global_static_cache_decode_fwd(h, cos, sin, pos, cache_k, cache_v, cache_length,
                                                wq, wk, wo, qn, kn)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["decode"] == n0 + 1
    assert int(cache_length) == length + 1
    untouched = torch.ones(cap, dtype=torch.bool)
    untouched[length] = False
    assert torch.equal(cache_k[:, :, untouched], before_k[:, :, untouched])
    assert torch.equal(cache_v[:, :, untouched], before_v[:, :, untouched])
    ref_out, ref_lse, k_new, v_new = _ref_layer(h, cos, sin, wq, wk, None, wo, qn, kn, cache_k,
                                                cache_v, length + 1, 32, 4, 512, None)
    assert rel_l2(cache_k[:, :, length].float().cpu(), k_new[0, 0].cpu()) < 1e-2
    assert rel_l2(cache_v[:, :, length].float().cpu(), v_new[0, 0].cpu()) < 1e-2
    assert out.shape == (1, 1, H) and lse.shape == (1, 32, 1)
    assert rel_l2(out.float().cpu(), ref_out.cpu()) < 2e-2
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) < 1e-3


@pytest.mark.parametrize("position", [700, 5000], ids=["filling", "rolling"])
@torch.no_grad()
def test_local_decode_step_fills_then_rolls_the_window(position):
    g = torch.Generator().manual_seed(2)
    h = torch.randn(1, 1, H, generator=g).bfloat16().cuda()
    cos, sin = _rope(g, 256)
    wq, wk, wv, wo, qn, kn = _weights(g, [(32 * 256, H), (16 * 256, H), (16 * 256, H),
                                          (H, 32 * 256), (256,), (256,)])
    filled = min(position, d.LOCAL_WINDOW)
    cache_k = torch.zeros(1, 16, d.LOCAL_WINDOW, 256, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    cache_k[:, :, :filled] = _rms_unit(torch.randn(1, 16, filled, 256, generator=g)).bfloat16().cuda()
    cache_v[:, :, :filled] = _rms_unit(torch.randn(1, 16, filled, 256, generator=g)).bfloat16().cuda()
    before_k, before_v = cache_k.clone(), cache_v.clone()
    cache_length = torch.tensor(filled, dtype=torch.int64, device="cuda")
    pos = torch.full((1, 1), position, dtype=torch.int64, device="cuda")
    out, lse = d.local_static_cache_decode_fwd(h, cos, sin, pos, cache_k, cache_v, cache_length,
                                               wq, wk, wv, wo, qn, kn)
    torch.cuda.synchronize()
    assert int(cache_length) == filled  # read only for the local op
    if position < d.LOCAL_WINDOW:
        slot, active = position, position + 1
        keep = torch.ones(d.LOCAL_WINDOW, dtype=torch.bool)
        keep[slot] = False
        assert torch.equal(cache_k[:, :, keep], before_k[:, :, keep])
        assert torch.equal(cache_v[:, :, keep], before_v[:, :, keep])
    else:
        slot, active = d.LOCAL_WINDOW - 1, d.LOCAL_WINDOW
        assert torch.equal(cache_k[:, :, :-1], before_k[:, :, 1:])
        assert torch.equal(cache_v[:, :, :-1], before_v[:, :, 1:])
    ref_out, ref_lse, k_new, v_new = _ref_layer(h, cos, sin, wq, wk, wv, wo, qn, kn, cache_k,
                                                cache_v, active, 32, 16, 256, 1024)
    assert rel_l2(cache_k[:, :, slot].float().cpu(), k_new[0, 0].cpu()) < 1e-2
    assert rel_l2(cache_v[:, :, slot].float().cpu(), v_new[0, 0].cpu()) < 1e-2
    assert rel_l2(out.float().cpu(), ref_out.cpu()) < 2e-2
    assert lse_abs_err(lse.cpu().numpy(), ref_lse) < 1e-3


@torch.no_grad()
def test_global_decode_refuses_a_full_cache_before_mutating_it():
    g = torch.Generator().manual_seed(3)
    cap = 64
    h = torch.randn(1, 1, H, generator=g).bfloat16().cuda()
    cos, sin = _rope(g, 512)
    ws = _weights(g, [(32 * 512, H), (4 * 512, H), (H, 32 * 512), (512,), (512,)])
    cache_k = torch.ones(1, 4, cap, 512, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.ones_like(cache_k)
    cache_length = torch.tensor(cap - 1, dtype=torch.int64, device="cuda")
    pos = torch.full((1, 1), cap - 1, dtype=torch.int64, device="cuda")
    from gemma4_fa4_kernels_b200 import UnsupportedB200Path

    with pytest.raises(UnsupportedB200Path, match="spare"):
        d.global_static_cache_decode_fwd(h, cos, sin, pos, cache_k, cache_v, cache_length, *ws)
    assert int(cache_length) == cap - 1 and bool((cache_k == 1).all())
