"""Float64 restatement of the Gemma-4 Q/K/V preparation (TEST INFRASTRUCTURE ONLY).

Forward, following the reference project:

* ``rms_norm`` -- ``x * (mean(x^2) + eps)^-1/2``, times an optional learned
  scale (``src/gemma4_fa4/reference.py:276-281``; the layer ops' FP32 order in
  ``src/gemma4_fa4/h100_torch_ops.py:302-313``);
* ``apply_partial_rotary`` -- rotate-half RoPE on the leading ``rotary_dim``
  features, the rest passed through (``reference.py:289-303``).  With
  ``rotary_dim == D`` this is the layer ops' ``_apply_rotary``
  (``h100_torch_ops.py:316-326``), whose proportional partial rotation is
  carried by cos = 1 / sin = 0 entries of a full-width table;
* ``prepare_global_kv`` -- K = partial_RoPE(KNorm(Z)), V = VNorm(Z) from one
  projection source Z (``reference.py:306-328``).

Backward: the analytic adjoints of the same maps (the reference gets them
from torch autograd, ``tests/test_reference.py:381-407``):

* RoPE^T: ``dn_j = g_j cos_j + g_{j+h} sin_{j+h}`` for ``j < h`` and
  ``dn_j = g_j cos_j - g_{j-h} sin_{j-h}`` for ``h <= j < 2h`` (h = rotary_dim/2);
* the learned scale: ``dw = sum over rows of dn * y``;
* RMS norm: ``dx = r * (dy - y * mean(dy * y))`` with ``y = x r``.

Arrays are (..., rows..., D); cos/sin broadcast against x[..., :rotary_dim]
exactly as the caller supplies them (already expanded by the caller).
"""

from __future__ import annotations

import numpy as np


def rms_norm(x, weight=None, eps=1e-6):
    x = np.asarray(x, dtype=np.float64)
    r = (np.mean(x * x, axis=-1, keepdims=True) + eps) ** -0.5
    y = x * r
    if weight is not None:
        y = y * np.asarray(weight, dtype=np.float64)
    return y


def apply_partial_rotary(x, cos, sin, rotary_dim):
    x = np.asarray(x, dtype=np.float64)
    if rotary_dim == 0:
        return x.copy()
    h = rotary_dim // 2
    xr = x[..., :rotary_dim]
    rot = np.concatenate((-xr[..., h:], xr[..., :h]), axis=-1)
    out = x.copy()
    out[..., :rotary_dim] = xr * cos + rot * sin
    return out


def rotary_adjoint(g, cos, sin, rotary_dim):
    """Transpose of ``apply_partial_rotary`` applied to the cotangent ``g``."""
    g = np.asarray(g, dtype=np.float64)
    if rotary_dim == 0:
        return g.copy()
    h = rotary_dim // 2
    gr = g[..., :rotary_dim]
    t = gr * sin
    out = g.copy()
    out[..., :rotary_dim] = gr * cos + np.concatenate((t[..., h:], -t[..., :h]), axis=-1)
    return out


def rotary_width(head_dim, partial_rotary_factor):
    width = head_dim * partial_rotary_factor
    if int(width) != width or int(width) % 2:
        raise ValueError("partial rotary width must be an even integer")
    return int(width)


def prepare_global_kv(source, k_norm_weight, cos, sin, partial_rotary_factor=0.25, eps=1e-6):
    rd = rotary_width(np.shape(source)[-1], partial_rotary_factor)
    k = apply_partial_rotary(rms_norm(source, k_norm_weight, eps), cos, sin, rd)
    v = rms_norm(source, None, eps)
    return k, v


def prepare_bwd(x, weight, cos, sin, rotary_dim, d_rot=None, d_plain=None, eps=1e-6):
    """Gradients of ``rot = RoPE(RMS(x) * weight)`` and ``plain = RMS(x)``.

    Returns ``(dx, dweight)``; ``dweight`` sums over every leading axis and is
    None when ``weight`` is None.  Either cotangent may be None (zero)."""
    x = np.asarray(x, dtype=np.float64)
    d = x.shape[-1]
    r = (np.mean(x * x, axis=-1, keepdims=True) + eps) ** -0.5
    y = x * r
    dy = np.zeros_like(x)
    dw = None
    if d_rot is not None:
        dn = rotary_adjoint(d_rot, cos, sin, rotary_dim)
        if weight is not None:
            w = np.asarray(weight, dtype=np.float64)
            dw = (dn * y).reshape(-1, d).sum(axis=0)
            dn = dn * w
        dy = dy + dn
    elif weight is not None:
        dw = np.zeros(d)
    if d_plain is not None:
        dy = dy + np.asarray(d_plain, dtype=np.float64)
    dx = r * (dy - y * np.mean(dy * y, axis=-1, keepdims=True))
    return dx, dw
