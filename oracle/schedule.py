"""Exact tile-incidence schedule for local metadata attention (test oracle).

The reference builds, per packed sequence, forward Q-tile -> K-tile candidate
lists and a transposed backward K-tile -> Q-tile list
(``src/gemma4_fa4/sparse_schedule.py:181-374``).  Its candidate set for a
tile pair is non-empty exactly when the tile pair holds at least one allowed
(q, k) under the complete Gemma local mask: the strict-left-window causal
band restricted to the query's document, plus same-(document, vision) keys
after the earliest query of that pair in the tile
(``sparse_schedule.py:205-266``).

This restatement computes that incidence directly from the index mask, one
tile pair at a time, which is quadratic and meant for small cases; the
storage bound follows ``sparse_schedule.py:94-125``.
"""

from __future__ import annotations

import numpy as np


def _ceildiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _incidence(vis, doc, *, q_length, k_length, q_block, k_block, window):
    q_off = k_length - q_length
    nq = _ceildiv(q_length, q_block)
    nk = _ceildiv(k_length, k_block)
    vis = np.asarray(vis, dtype=np.int64)
    doc = np.asarray(doc, dtype=np.int64)
    rows = []
    kk_all = np.arange(k_length, dtype=np.int64)
    for qb in range(nq):
        qa = np.arange(q_off + qb * q_block, q_off + min(q_length, (qb + 1) * q_block), dtype=np.int64)
        allowed = kk_all[None, :] <= qa[:, None]
        qv = vis[qa]
        allowed |= (qv[:, None] == vis[None, :]) & (qv[:, None] >= 0)
        allowed &= kk_all[None, :] > qa[:, None] - window
        allowed &= doc[qa][:, None] == doc[None, :]
        col_any = allowed.any(axis=0)
        hit = [kb for kb in range(nk) if col_any[kb * k_block:(kb + 1) * k_block].any()]
        rows.append(tuple(hit))
    return rows, nk


def _transpose(rows, n_cols):
    out = [[] for _ in range(n_cols)]
    for r, cols in enumerate(rows):
        for c in cols:
            out[c].append(r)
    return [tuple(x) for x in out]


def _storage_bytes(rows):
    width = max([1] + [len(r) for r in rows])
    return 4 * len(rows) * (3 + width)


def build_local_sparse_schedule(vision_block_ids, document_ids, *, q_length, k_length,
                                sliding_window=1024, forward_block_size=(128, 80),
                                backward_block_size=(64, 64)):
    """Return a dict with ``forward`` rows (per Q tile), ``backward`` rows
    (per K tile, listing Q tiles of ``backward_block_size``) and the compact
    storage bytes of each, matching ``build_gemma4_local_sparse_schedule``."""
    if q_length <= 0 or k_length <= 0 or q_length > k_length:
        raise ValueError("sparse scheduling requires 1 <= Sq <= Sk")
    if len(vision_block_ids) != k_length or len(document_ids) != k_length:
        raise ValueError("vision/document metadata must match Sk")
    fwd, _ = _incidence(vision_block_ids, document_ids, q_length=q_length, k_length=k_length,
                        q_block=forward_block_size[0], k_block=forward_block_size[1],
                        window=sliding_window)
    bq, bk = backward_block_size
    bwd_q2k, nk = _incidence(vision_block_ids, document_ids, q_length=q_length,
                             k_length=k_length, q_block=bq, k_block=bk, window=sliding_window)
    bwd = _transpose(bwd_q2k, nk)
    return {
        "forward": fwd,
        "backward": bwd,
        "forward_storage_bytes": _storage_bytes(fwd),
        "backward_storage_bytes": _storage_bytes(bwd),
    }


def local_sparse_storage_upper_bound(q_length, k_length, *, forward_block_size=(128, 80),
                                     backward_block_size=(64, 64)):
    """Worst-case compact bytes, forward plus transposed backward
    (``sparse_schedule.py:94-125``)."""
    if q_length <= 0 or k_length <= 0 or q_length > k_length:
        raise ValueError("sparse scheduling requires 1 <= Sq <= Sk")
    f = 4 * _ceildiv(q_length, forward_block_size[0]) * (3 + _ceildiv(k_length, forward_block_size[1]))
    b = 4 * _ceildiv(k_length, backward_block_size[1]) * (3 + _ceildiv(q_length, backward_block_size[0]))
    return f + b
