"""High-precision Gemma-4 attention forward/backward in numpy (test oracle).

Restates ``src/gemma4_fa4/reference.py`` of the reference project:

* ``attention_fwd``  <- ``reference_attention`` (``reference.py:23-75``):
  scale 1.0 by default, GQA by repeating each KV head over its query group,
  masked scores set to -inf, natural-log LSE, fully masked rows give O = 0 and
  LSE = -inf.
* ``attention_bwd``  <- the autograd of the same expression (the reference
  differentiates ``reference_attention`` with torch autograd).  Written out:
  ``dV = P^T dO``, ``dP = dO V^T``, ``dS = P * (dP - rowsum(dO*O) + dLSE)``,
  ``dQ = scale * dS K``, ``dK = scale * dS^T Q``; GQA gradients are summed
  over each KV head's query group.
* ``attention_fwd_varlen`` <- ``reference_attention_varlen``
  (``reference.py:96-198``): per-segment lower-right loop over ``cu_seqlens``,
  metadata read along the packed K stream, empty-Q segments skipped.
* ``valid_pair_count`` / ``attention_flops`` <- ``reference.py:331-356``.

Tensors use the reference's ``(B, H, S, D)`` layout.  All arithmetic is
float64 unless ``dtype`` says otherwise; heads are processed one at a time so
that only one ``(Sq, Sk)`` score matrix is alive.
"""

from __future__ import annotations

import numpy as np

from .masks import gemma4_attention_mask


def _mask(b, q_len, kv_len, *, sliding_window, vision_block_ids, document_ids,
          key_padding_mask, allow_vision_bidirectional, q_start):
    return gemma4_attention_mask(
        batch_size=b,
        q_len=q_len,
        kv_len=kv_len,
        sliding_window=sliding_window,
        vision_block_ids=vision_block_ids,
        document_ids=document_ids,
        key_padding_mask=key_padding_mask,
        q_start=q_start,
        allow_vision_bidirectional=allow_vision_bidirectional,
    )[:, 0]


def _check(q, k, v):
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k, and v must be rank-4 B/H/S/D arrays")
    b, hq, _, d = q.shape
    bk, hkv, kv_len, dk = k.shape
    bv, hv, vv_len, _ = v.shape
    if (bk, bv) != (b, b) or hkv != hv or kv_len != vv_len or d != dk:
        raise ValueError("incompatible q/k/v shapes")
    if hq % hkv:
        raise ValueError("query heads must be divisible by KV heads")
    return hq // hkv


def _head_probs(scores, allowed):
    """Masked softmax of one head: returns (P, lse) with the reference's
    fully-masked-row convention (P = 0, lse = -inf)."""
    s = np.where(allowed, scores, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    finite = np.isfinite(m)
    m_safe = np.where(finite, m, 0.0)
    e = np.exp(s - m_safe)
    denom = e.sum(axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        lse = np.where(finite, m_safe + np.log(denom), -np.inf)[..., 0]
        p = np.where(finite, e / np.where(finite, denom, 1.0), 0.0)
    return p, lse


def attention_fwd(
    q, k, v, *,
    softmax_scale: float = 1.0,
    sliding_window: int | None = None,
    vision_block_ids=None,
    document_ids=None,
    key_padding_mask=None,
    allow_vision_bidirectional: bool = False,
    q_start: int | None = None,
    dtype=np.float64,
):
    """Return ``(out, lse)``: out ``(B,Hq,Sq,Dv)`` in ``dtype``, lse
    ``(B,Hq,Sq)`` float32 (``reference.py:23-75``)."""
    rep = _check(q, k, v)
    b, hq, q_len, _ = q.shape
    kv_len = k.shape[2]
    allowed = _mask(b, q_len, kv_len, sliding_window=sliding_window,
                    vision_block_ids=vision_block_ids, document_ids=document_ids,
                    key_padding_mask=key_padding_mask,
                    allow_vision_bidirectional=allow_vision_bidirectional, q_start=q_start)
    qf, kf, vf = (np.asarray(x, dtype=dtype) for x in (q, k, v))
    out = np.zeros((b, hq, q_len, v.shape[-1]), dtype=dtype)
    lse = np.zeros((b, hq, q_len), dtype=np.float64)
    for bi in range(b):
        for h in range(hq):
            hk = h // rep
            scores = (qf[bi, h] @ kf[bi, hk].T) * dtype(softmax_scale)
            p, l_ = _head_probs(scores, allowed[bi])
            out[bi, h] = p @ vf[bi, hk]
            lse[bi, h] = l_
    return out, lse.astype(np.float32)


def attention_bwd(
    q, k, v, dout, *,
    dlse=None,
    softmax_scale: float = 1.0,
    sliding_window: int | None = None,
    vision_block_ids=None,
    document_ids=None,
    key_padding_mask=None,
    allow_vision_bidirectional: bool = False,
    q_start: int | None = None,
    dtype=np.float64,
):
    """Return ``(dq, dk, dv)`` of ``attention_fwd`` for upstream ``dout``
    (and optional ``dlse``), in ``dtype``."""
    rep = _check(q, k, v)
    b, hq, q_len, _ = q.shape
    hkv, kv_len = k.shape[1], k.shape[2]
    allowed = _mask(b, q_len, kv_len, sliding_window=sliding_window,
                    vision_block_ids=vision_block_ids, document_ids=document_ids,
                    key_padding_mask=key_padding_mask,
                    allow_vision_bidirectional=allow_vision_bidirectional, q_start=q_start)
    qf, kf, vf, dof = (np.asarray(x, dtype=dtype) for x in (q, k, v, dout))
    dlf = None if dlse is None else np.asarray(dlse, dtype=dtype)
    scale = dtype(softmax_scale)
    dq = np.zeros_like(qf)
    dk = np.zeros((b, hkv, kv_len, k.shape[-1]), dtype=dtype)
    dv = np.zeros((b, hkv, kv_len, v.shape[-1]), dtype=dtype)
    for bi in range(b):
        for h in range(hq):
            hk = h // rep
            scores = (qf[bi, h] @ kf[bi, hk].T) * scale
            p, _ = _head_probs(scores, allowed[bi])
            o = p @ vf[bi, hk]
            dp = dof[bi, h] @ vf[bi, hk].T
            delta = (dof[bi, h] * o).sum(axis=-1, keepdims=True)
            ds = p * (dp - delta)
            if dlf is not None:
                ds = ds + p * np.where(np.isfinite(dlf[bi, h]), dlf[bi, h], 0.0)[:, None]
            dv[bi, hk] += p.T @ dof[bi, h]
            dq[bi, h] = (ds @ kf[bi, hk]) * scale
            dk[bi, hk] += (ds.T @ qf[bi, h]) * scale
    return dq, dk, dv


def _cumulative(cu, total, name):
    values = [int(x) for x in np.asarray(cu).tolist()]
    if len(values) < 2:
        raise ValueError(f"{name} must be rank-1 with at least two entries")
    if values[0] != 0 or values[-1] != total:
        raise ValueError(f"{name} must start at zero and end at the packed total")
    if any(e < s for s, e in zip(values[:-1], values[1:])):
        raise ValueError(f"{name} must be nondecreasing")
    return values


def _segments(q, k, cu_q, cu_k):
    qc = _cumulative(cu_q, q.shape[0], "cu_seqlens_q")
    kc = _cumulative(cu_k, k.shape[0], "cu_seqlens_k")
    if len(qc) != len(kc):
        raise ValueError("packed Q and K must have the same batch count")
    segs = []
    for i, (qs, qe, ks, ke) in enumerate(zip(qc[:-1], qc[1:], kc[:-1], kc[1:])):
        if qe - qs > ke - ks:
            raise ValueError(f"packed sequence {i} has Sq greater than Sk")
        segs.append((qs, qe, ks, ke))
    return segs


def _seg_meta(meta, ks, ke):
    return None if meta is None else np.asarray(meta)[ks:ke][None, :]


def attention_fwd_varlen(
    q, k, v, cu_seqlens_q, cu_seqlens_k, *,
    softmax_scale: float = 1.0,
    sliding_window: int | None = None,
    vision_block_ids=None,
    document_ids=None,
    allow_vision_bidirectional: bool = False,
    dtype=np.float64,
):
    """Packed ``(T,H,D)`` forward (``reference.py:96-198``).  Returns
    ``(out (Tq,Hq,Dv), lse (Hq,Tq))``; rows of empty segments do not exist."""
    out = np.zeros((q.shape[0], q.shape[1], v.shape[-1]), dtype=dtype)
    lse = np.zeros((q.shape[1], q.shape[0]), dtype=np.float32)
    for qs, qe, ks, ke in _segments(q, k, cu_seqlens_q, cu_seqlens_k):
        if qe == qs:
            continue
        o, l_ = attention_fwd(
            np.asarray(q)[qs:qe].transpose(1, 0, 2)[None],
            np.asarray(k)[ks:ke].transpose(1, 0, 2)[None],
            np.asarray(v)[ks:ke].transpose(1, 0, 2)[None],
            softmax_scale=softmax_scale, sliding_window=sliding_window,
            vision_block_ids=_seg_meta(vision_block_ids, ks, ke),
            document_ids=_seg_meta(document_ids, ks, ke),
            allow_vision_bidirectional=allow_vision_bidirectional,
            q_start=(ke - ks) - (qe - qs), dtype=dtype,
        )
        out[qs:qe] = o[0].transpose(1, 0, 2)
        lse[:, qs:qe] = l_[0]
    return out, lse


def attention_fwd_bwd_varlen(
    q, k, v, dout, cu_seqlens_q, cu_seqlens_k, *,
    dlse=None,
    softmax_scale: float = 1.0,
    sliding_window: int | None = None,
    vision_block_ids=None,
    document_ids=None,
    allow_vision_bidirectional: bool = False,
    dtype=np.float64,
):
    """Packed forward plus gradients; empty-Q segments give exact-zero K/V
    gradients (``test_reference.py:140-179``).  Returns
    ``(out, lse, dq, dk, dv)`` in packed layouts."""
    out, lse = attention_fwd_varlen(
        q, k, v, cu_seqlens_q, cu_seqlens_k, softmax_scale=softmax_scale,
        sliding_window=sliding_window, vision_block_ids=vision_block_ids,
        document_ids=document_ids, allow_vision_bidirectional=allow_vision_bidirectional,
        dtype=dtype)
    dq = np.zeros(q.shape, dtype=dtype)
    dk = np.zeros(k.shape, dtype=dtype)
    dv = np.zeros(v.shape, dtype=dtype)
    for qs, qe, ks, ke in _segments(q, k, cu_seqlens_q, cu_seqlens_k):
        if qe == qs:
            continue
        tr = lambda x: np.asarray(x).transpose(1, 0, 2)[None]  # noqa: E731
        g = attention_bwd(
            tr(np.asarray(q)[qs:qe]), tr(np.asarray(k)[ks:ke]), tr(np.asarray(v)[ks:ke]),
            tr(np.asarray(dout)[qs:qe]),
            dlse=None if dlse is None else np.asarray(dlse)[:, qs:qe][None],
            softmax_scale=softmax_scale, sliding_window=sliding_window,
            vision_block_ids=_seg_meta(vision_block_ids, ks, ke),
            document_ids=_seg_meta(document_ids, ks, ke),
            allow_vision_bidirectional=allow_vision_bidirectional,
            q_start=(ke - ks) - (qe - qs), dtype=dtype,
        )
        dq[qs:qe] = g[0][0].transpose(1, 0, 2)
        dk[ks:ke] = g[1][0].transpose(1, 0, 2)
        dv[ks:ke] = g[2][0].transpose(1, 0, 2)
    return out, lse, dq, dk, dv


def valid_pair_count(seqlen: int, sliding_window: int | None) -> int:
    """Text-only causal(+window) pair count (``reference.py:331-335``)."""
    if sliding_window is None:
        return seqlen * (seqlen + 1) // 2
    w = min(sliding_window, seqlen)
    return seqlen * w - w * (w - 1) // 2


def attention_flops(*, num_q_heads, head_dim_qk, head_dim_v, batch, seqlen,
                    sliding_window, mode="fwd", pairs=None):
    """Matmul FLOPs (``reference.py:338-356``).  ``pairs`` overrides the
    text-only pair count with an exact mask-aware count (summed over the
    batch, so ``batch`` is then ignored)."""
    if pairs is None:
        pairs = batch * valid_pair_count(seqlen, sliding_window)
    fwd = 2.0 * num_q_heads * pairs * (head_dim_qk + head_dim_v)
    bwd = 2.0 * num_q_heads * pairs * (3 * head_dim_qk + 2 * head_dim_v)
    if mode == "fwd":
        return fwd
    if mode == "bwd":
        return bwd
    if mode == "fwd_bwd":
        return fwd + bwd
    raise ValueError(mode)


def mask_aware_pairs(*, q_len, kv_len, sliding_window, vision_block_ids=None,
                     document_ids=None, allow_vision_bidirectional=False, chunk=2048):
    """Exact count of allowed (q, k) pairs of one sequence under the full
    Gemma mask, computed in row chunks so long sequences stay bounded."""
    total = 0
    q_off = kv_len - q_len
    vis = None if vision_block_ids is None else np.asarray(vision_block_ids).reshape(-1)
    doc = None if document_ids is None else np.asarray(document_ids).reshape(-1)
    kk = np.arange(kv_len, dtype=np.int64)
    for r0 in range(0, q_len, chunk):
        r1 = min(q_len, r0 + chunk)
        qa = np.arange(r0 + q_off, r1 + q_off, dtype=np.int64)
        allowed = kk[None, :] <= qa[:, None]
        if vis is not None and allow_vision_bidirectional:
            qv = vis[qa]
            allowed |= (qv[:, None] == vis[None, :]) & (qv[:, None] >= 0)
        if sliding_window is not None:
            allowed &= kk[None, :] > qa[:, None] - sliding_window
        if doc is not None:
            allowed &= doc[qa][:, None] == doc[None, :]
        total += int(allowed.sum())
    return total
