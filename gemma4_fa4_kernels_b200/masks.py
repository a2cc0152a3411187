"""Exact index-level Gemma-4 attention masks (``src/gemma4_fa4/masks.py:8-86``).

``gemma4_attention_mask`` returns the allowed-position bool mask ``(B, 1, Q, K)``:
causal with lower-right query alignment, OR (sliding layers with
``allow_vision_bidirectional``) the same non-negative vision block, AND the
strict window ``k > q - W``, AND the same document, AND key padding.

On a CUDA device the mask is produced by the library kernel
(``g4_build_mask``).  On a CPU device (host-side mask planning, as the
Transformers integration does) it is built with torch index arithmetic; the
attention kernels never consume dense masks.
"""

from __future__ import annotations

import torch

from . import ops


def _check_meta(values, batch_size, kv_len, name):
    if values is not None and tuple(values.shape) != (batch_size, kv_len):
        raise ValueError(f"{name} must be {(batch_size, kv_len)}, got {tuple(values.shape)}")


def gemma4_attention_mask(
    *,
    batch_size: int,
    q_len: int,
    kv_len: int,
    device: torch.device | str,
    sliding_window: int | None,
    vision_block_ids: torch.Tensor | None = None,
    document_ids: torch.Tensor | None = None,
    key_padding_mask: torch.Tensor | None = None,
    q_start: int | None = None,
    allow_vision_bidirectional: bool = False,
) -> torch.Tensor:
    """Bool mask ``(B, 1, Q, K)``; True means the (query, key) pair is allowed."""
    if batch_size < 1 or q_len < 0 or kv_len < 0:
        raise ValueError("invalid attention shape")
    if q_len > kv_len and q_start is None:
        raise ValueError("q_len cannot exceed kv_len when q_start is omitted")
    if sliding_window is not None and sliding_window <= 0:
        raise ValueError("sliding_window must be positive")
    start = kv_len - q_len if q_start is None else q_start
    if start < 0 or start + q_len > kv_len:
        raise ValueError("query positions must lie inside the KV stream")
    _check_meta(vision_block_ids, batch_size, kv_len, "vision_block_ids")
    _check_meta(document_ids, batch_size, kv_len, "document_ids")
    _check_meta(key_padding_mask, batch_size, kv_len, "key_padding_mask")
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    use_vision = vision_block_ids is not None and allow_vision_bidirectional

    if device.type == "cuda":
        m = ops.build_mask(batch_size, q_len, kv_len, window=sliding_window or 0,
                           allow_vision_bidirectional=use_vision,
                           vision_ids=vision_block_ids.to(device) if use_vision else None,
                           document_ids=None if document_ids is None else document_ids.to(device),
                           key_padding_mask=None if key_padding_mask is None
                           else key_padding_mask.to(device),
                           q_start=start, device=device)
        return m.to(torch.bool)[:, None]

    qi = torch.arange(start, start + q_len, device=device)
    ki = torch.arange(kv_len, device=device)
    allowed = (ki[None, :] <= qi[:, None]).expand(batch_size, q_len, kv_len).clone()
    if use_vision:
        vb = vision_block_ids.to(device)
        qb = vb[:, qi]
        allowed |= (qb[:, :, None] == vb[:, None, :]) & (qb[:, :, None] >= 0)
    if sliding_window is not None:
        allowed &= (ki[None, :] > qi[:, None] - sliding_window)[None]
    if document_ids is not None:
        db = document_ids.to(device)
        allowed &= db[:, qi][:, :, None] == db[:, None, :]
    if key_padding_mask is not None:
        allowed &= key_padding_mask.to(device=device, dtype=torch.bool)[:, None, :]
    return allowed[:, None]


def additive_mask(mask: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Allowed-position bool mask to a 0 / -inf additive mask."""
    out = torch.zeros(mask.shape, dtype=dtype, device=mask.device)
    return out.masked_fill(~mask, float("-inf"))
