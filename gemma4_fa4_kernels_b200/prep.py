"""Fused Q/K/V preparation: RMS norm, learned scale and rotate-half RoPE in one
pass, with autograd through the fused adjoint (``g4_prep_fwd`` / ``g4_prep_bwd``).

Gemma-4 prepares the attention operands from the projections as

* ``Q = RoPE(QNorm(q_proj(h)))``, ``K = RoPE(KNorm(k_proj(h)))``,
  ``V = VNorm(v_proj(h))`` (``src/gemma4_fa4/h100_torch_ops.py:396-403``);
* global layers: ``Z = k_proj(h)``, ``K = partial_RoPE(KNorm(Z))``,
  ``V = VNorm(Z)`` (``reference.py:306-328``, ``h100_torch_ops.py:456-461``).

``KNorm``/``QNorm`` carry a learned scale; ``VNorm`` has none.  The shared
source form reads Z once and writes K and V; its backward applies the
K-side adjoint (RoPE^T, scale, norm) and the V-side norm adjoint and sums
them into dZ -- not ``dK + dV`` (``docs/design.md:202-213``).

Operands are BF16.  Layouts: ``"bshd"`` (B, S, H, D) with tables (B or 1, S,
R) -- the layer ops' order (rotary before the head transpose); ``"bhsd"``
(B, H, S, D) with tables (B or 1, S, R) -- the reference helper's broadcast;
``"thd"`` packed (T, H, D) with tables (T, R).  The tables cover the leading
R features; full-width (R = D) tables reproduce the layer ops, whose
proportional partial rotation lives in cos = 1 / sin = 0 entries.  Head dims
256 and 512; R zero or a power of two >= 16 (Gemma-4: 128, 256, 512).  There is no CPU path: without the native
library every call raises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .errors import UnsupportedB200Path
from .ops import _raise_for, _stream, _workspace

RMS_EPS = 1e-6
LAYOUTS = ("bshd", "bhsd", "thd")


def _geometry(x: torch.Tensor, layout: str):
    """(batch, seqlen, heads, [batch, token, head] strides) of a prep operand."""
    if layout == "bshd":
        b, s, h, _ = x.shape
        return b, s, h, (x.stride(0), x.stride(1), x.stride(2))
    if layout == "bhsd":
        b, h, s, _ = x.shape
        return b, s, h, (x.stride(0), x.stride(2), x.stride(1))
    t, h, _ = x.shape
    return 1, t, h, (0, x.stride(0), x.stride(1))


def _arr(vals, n=3):
    a = (ctypes.c_int64 * n)()
    for i, v in enumerate(vals):
        a[i] = int(v)
    return a


def _check_operand(x: torch.Tensor, layout: str, what: str) -> None:
    if layout not in LAYOUTS:
        raise ValueError(f"layout must be one of {LAYOUTS}")
    if x.ndim != (3 if layout == "thd" else 4):
        raise ValueError(f"{what} must be rank {3 if layout == 'thd' else 4} for layout {layout}")
    if x.device.type != "cuda":
        raise UnsupportedB200Path(f"{what} must be a CUDA tensor")
    if x.dtype != torch.bfloat16:
        raise UnsupportedB200Path(f"{what} must be BF16")
    if x.stride(-1) != 1:
        raise ValueError(f"{what} must have unit stride along the head dimension")


def _tables(cos, sin, x, layout, rotary_dim):
    """BF16 tables with unit feature stride and their [batch, token] strides."""
    if rotary_dim == 0:
        return None, None, (0, 0)
    b, s, _, _ = _geometry(x, layout)
    want = (s, rotary_dim) if layout == "thd" else None
    out = []
    for name, t in (("cos", cos), ("sin", sin)):
        if t is None:
            raise ValueError(f"{name} is required when the rotary width is nonzero")
        if t.device != x.device:
            raise ValueError(f"{name} must be on the operand device")
        t = t.to(torch.bfloat16)
        if t.stride(-1) != 1 or t.data_ptr() % 16 or any(st % 8 for st in t.stride()[:-1]):
            t = t.contiguous()
        if layout == "thd":
            if tuple(t.shape) != want:
                raise ValueError(f"{name} must be (T, {rotary_dim}) for packed operands")
        elif t.ndim != 3 or t.shape[0] not in (1, b) or t.shape[1] != s or t.shape[2] != rotary_dim:
            raise ValueError(f"{name} must be (B or 1, S, {rotary_dim}); got {tuple(t.shape)}")
        out.append(t)
    c, sn = out
    if c.stride() != sn.stride():
        c, sn = c.contiguous(), sn.contiguous()
    if layout == "thd":
        st = (0, c.stride(0))
    else:
        st = (0 if c.shape[0] == 1 else c.stride(0), c.stride(1))
    return c, sn, st


def _weight(weight, x):
    if weight is None:
        return None
    if weight.device != x.device:
        raise ValueError("norm weight must be on the operand device")
    if weight.dtype != torch.bfloat16:
        raise UnsupportedB200Path("norm weight must be BF16")
    if weight.shape != (x.shape[-1],):
        raise ValueError(f"norm weight must have shape ({x.shape[-1]},)")
    return weight.contiguous()


def prep_fwd(x, weight, cos, sin, rotary_dim, *, layout="bshd", eps=RMS_EPS, want_rot=True,
             want_plain=False):
    """``(RoPE(Norm(x) * weight) or None, Norm(x) or None)`` through ``g4_prep_fwd``."""
    _check_operand(x, layout, "x")
    w = _weight(weight, x)
    c, s, cst = _tables(cos, sin, x, layout, rotary_dim if want_rot else 0)
    b, sl, h, xst = _geometry(x, layout)
    rot = torch.empty_like(x) if want_rot else None
    plain = torch.empty_like(x) if want_plain else None
    if x.numel() == 0:
        return rot, plain
    a = _lib.G4PrepArgs()
    a.x, a.weight = x.data_ptr(), None if w is None else w.data_ptr()
    a.cos, a.sin = (None, None) if c is None else (c.data_ptr(), s.data_ptr())
    a.rot = None if rot is None else rot.data_ptr()
    a.plain = None if plain is None else plain.data_ptr()
    a.x_stride = _arr(xst)
    if rot is not None:
        a.rot_stride = _arr(_geometry(rot, layout)[3])
    if plain is not None:
        a.plain_stride = _arr(_geometry(plain, layout)[3])
    a.cos_stride = _arr(cst, 2)
    a.batch, a.seqlen, a.num_heads = b, sl, h
    a.head_dim, a.rotary_dim, a.eps = x.shape[-1], rotary_dim if want_rot else 0, float(eps)
    _raise_for(_lib.load().g4_prep_fwd(ctypes.byref(a), _stream(x.device)), "g4_prep_fwd")
    return rot, plain


def prep_bwd(x, weight, cos, sin, rotary_dim, drot, dplain, *, layout="bshd", eps=RMS_EPS,
             need_dweight=True):
    """``(dx, dweight float32 or None)`` through ``g4_prep_bwd``."""
    _check_operand(x, layout, "x")
    w = _weight(weight, x)
    if drot is None and dplain is None:
        raise ValueError("at least one cotangent is required")
    grads = []
    for name, g in (("drot", drot), ("dplain", dplain)):
        if g is None:
            grads.append(None)
            continue
        if g.shape != x.shape:
            raise ValueError(f"{name} must have the shape of x")
        g = g.to(torch.bfloat16)
        if g.stride(-1) != 1 or g.data_ptr() % 16 or any(st % 8 for st in g.stride()[:-1]):
            g = g.contiguous()
        grads.append(g)
    drot, dplain = grads
    rd = rotary_dim if drot is not None else 0
    c, s, cst = _tables(cos, sin, x, layout, rd)
    b, sl, h, xst = _geometry(x, layout)
    dx = torch.empty_like(x)
    want_dw = need_dweight and w is not None and drot is not None
    dw = torch.empty(x.shape[-1], dtype=torch.float32, device=x.device) if want_dw else None
    if x.numel() == 0:
        return dx, None if dw is None else dw.zero_()
    a = _lib.G4PrepArgs()
    a.x, a.weight = x.data_ptr(), None if w is None else w.data_ptr()
    a.cos, a.sin = (None, None) if c is None else (c.data_ptr(), s.data_ptr())
    a.drot = None if drot is None else drot.data_ptr()
    a.dplain = None if dplain is None else dplain.data_ptr()
    a.dx, a.dweight = dx.data_ptr(), None if dw is None else dw.data_ptr()
    a.x_stride = _arr(xst)
    if drot is not None:
        a.drot_stride = _arr(_geometry(drot, layout)[3])
    if dplain is not None:
        a.dplain_stride = _arr(_geometry(dplain, layout)[3])
    a.dx_stride = _arr(_geometry(dx, layout)[3])
    a.cos_stride = _arr(cst, 2)
    a.batch, a.seqlen, a.num_heads = b, sl, h
    a.head_dim, a.rotary_dim, a.eps = x.shape[-1], rd, float(eps)
    lib = _lib.load()
    ws = None
    need = lib.g4_prep_bwd_workspace_bytes(ctypes.byref(a))
    if need:
        ws = _workspace(need, x.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _raise_for(lib.g4_prep_bwd(ctypes.byref(a), _stream(x.device)), "g4_prep_bwd")
    return dx, dw


class _PrepFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, cos, sin, rotary_dim, layout, eps, want_rot, want_plain):
        rot, plain = prep_fwd(x, weight, cos, sin, rotary_dim, layout=layout, eps=eps,
                              want_rot=want_rot, want_plain=want_plain)
        ctx.save_for_backward(x, weight, cos, sin)
        ctx.cfg = (rotary_dim, layout, eps)
        ctx.set_materialize_grads(False)
        return rot, plain

    @staticmethod
    def backward(ctx, drot, dplain):
        x, weight, cos, sin = ctx.saved_tensors
        rotary_dim, layout, eps = ctx.cfg
        if drot is None and dplain is None:
            return (None,) * 9
        need_dw = weight is not None and ctx.needs_input_grad[1]
        dx, dw = prep_bwd(x, weight, cos, sin, rotary_dim, drot, dplain, layout=layout, eps=eps,
                          need_dweight=need_dw)
        if need_dw and dw is None:  # no rotated cotangent: the scale got no gradient
            dw = torch.zeros(x.shape[-1], dtype=torch.float32, device=x.device)
        return (dx, None if dw is None else dw.to(weight.dtype), None, None, None, None, None,
                None, None)


def _rotary_width(cos, head_dim):
    return 0 if cos is None else int(cos.shape[-1])


def prepare_rotary_operand(x, norm_weight, cos, sin, *, layout="bshd", eps=RMS_EPS):
    """``RoPE(Norm(x) * norm_weight)``: Q of every layer, K of local layers.

    Tables (B or 1, S, R) rotate the leading R features (R = D reproduces the
    layer ops' ``_apply_rotary`` on full-width tables)."""
    rd = _rotary_width(cos, x.shape[-1])
    rot, _ = _PrepFunction.apply(x, norm_weight, cos, sin, rd, layout, eps, True, False)
    return rot


def prepare_value(x, *, layout="bshd", eps=RMS_EPS):
    """``Norm(x)`` without scale or rotation: V of local layers."""
    _, plain = _PrepFunction.apply(x, None, None, None, 0, layout, eps, False, True)
    return plain


def prepare_shared_kv(source, k_norm_weight, cos, sin, *, layout="bshd", eps=RMS_EPS):
    """Global layers: ``K = RoPE(KNorm(Z))``, ``V = VNorm(Z)`` from one read of Z."""
    rd = _rotary_width(cos, source.shape[-1])
    k, v = _PrepFunction.apply(source, k_norm_weight, cos, sin, rd, layout, eps, True, True)
    return k, v


def prepare_global_kv_from_projection_source(source, *, k_norm_weight, cos, sin,
                                             partial_rotary_factor=0.25, eps=RMS_EPS,
                                             layout="bhsd"):
    """Drop-in for ``reference.prepare_global_kv_from_projection_source``
    (``reference.py:306-328``): same keywords, same ``ValueError`` for a
    rotary width that is not an even integer, same (B, H, S, D) source with
    (B, S, R) tables by default.  Returns distinct ``(k, v)``."""
    rotary_width = source.shape[-1] * partial_rotary_factor
    if int(rotary_width) != rotary_width or int(rotary_width) % 2:
        raise ValueError("partial rotary width must be an even integer")
    rd = int(rotary_width)
    if rd and cos is not None and cos.shape[-1] != rd:
        raise ValueError(f"cos/sin must cover the {rd} rotated features")
    k, v = _PrepFunction.apply(source, k_norm_weight, cos, sin, rd, layout, eps, True, True)
    return k, v
