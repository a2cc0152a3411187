"""Index-level Gemma-4 attention mask, restated in numpy (test oracle).

Follows ``src/gemma4_fa4/masks.py:8-80`` of the reference:

* causal ``k <= q`` with lower-right query alignment (``q_start = Sk - Sq``);
* OR, on sliding layers with ``allow_vision_bidirectional``, the same
  non-negative vision block (no right cap);
* AND the strict left window ``k > q - W``;
* AND the same document;
* AND key padding.
"""

from __future__ import annotations

import numpy as np


def gemma4_attention_mask(
    *,
    batch_size: int,
    q_len: int,
    kv_len: int,
    sliding_window: int | None,
    vision_block_ids: np.ndarray | None = None,
    document_ids: np.ndarray | None = None,
    key_padding_mask: np.ndarray | None = None,
    q_start: int | None = None,
    allow_vision_bidirectional: bool = False,
) -> np.ndarray:
    """Bool mask ``(B, 1, Q, K)``; True = allowed (``masks.py:8-80``)."""
    if batch_size < 1 or q_len < 0 or kv_len < 0:
        raise ValueError("invalid attention shape")
    if q_len > kv_len and q_start is None:
        raise ValueError("q_len cannot exceed kv_len when q_start is omitted")
    if sliding_window is not None and sliding_window <= 0:
        raise ValueError("sliding_window must be positive")
    q_start = kv_len - q_len if q_start is None else q_start
    if q_start < 0 or q_start + q_len > kv_len:
        raise ValueError("query positions must lie inside the KV stream")

    q_idx = np.arange(q_start, q_start + q_len, dtype=np.int64)
    k_idx = np.arange(kv_len, dtype=np.int64)
    allowed = np.broadcast_to(k_idx[None, :] <= q_idx[:, None], (batch_size, q_len, kv_len)).copy()

    if vision_block_ids is not None:
        vision_block_ids = np.asarray(vision_block_ids)
        if vision_block_ids.shape != (batch_size, kv_len):
            raise ValueError("vision_block_ids must be (B, K)")
        if allow_vision_bidirectional:
            qb = vision_block_ids[:, q_idx]
            allowed |= (qb[:, :, None] == vision_block_ids[:, None, :]) & (qb[:, :, None] >= 0)

    if sliding_window is not None:
        allowed &= (k_idx[None, :] > q_idx[:, None] - sliding_window)[None]

    if document_ids is not None:
        document_ids = np.asarray(document_ids)
        if document_ids.shape != (batch_size, kv_len):
            raise ValueError("document_ids must be (B, K)")
        qd = document_ids[:, q_idx]
        allowed &= qd[:, :, None] == document_ids[:, None, :]

    if key_padding_mask is not None:
        key_padding_mask = np.asarray(key_padding_mask).astype(bool)
        if key_padding_mask.shape != (batch_size, kv_len):
            raise ValueError("key_padding_mask must be (B, K)")
        allowed &= key_padding_mask[:, None, :]

    return allowed[:, None, :, :]
