"""The reference's CPU attention in torch (TEST AND CPU-BASELINE INFRASTRUCTURE).

Restates ``reference_attention`` (``src/gemma4_fa4/reference.py:23-75``) as
the reference computes it: operands upcast to ``upcast`` (float64 by default,
float32 as the reference's ``upcast=torch.float32`` option), the KV heads
repeated over their query group, ``einsum`` scores, ``masked_fill(-inf)``
with the exact Gemma mask, ``logsumexp``, probabilities zeroed on fully
masked rows, ``einsum`` output; gradients by torch autograd
(``out.backward(dO)``), as the reference's tests and benchmark ruler do.

``bench.py`` times it on the host cores as the CPU baseline; the float64 numpy
oracle in ``attention.py`` is the parity pin (both restate the same function).
"""

from __future__ import annotations

import numpy as np
import torch

from .masks import gemma4_attention_mask


def reference_attention_torch(q, k, v, *, sliding_window=None, vision_block_ids=None,
                              document_ids=None, allow_vision_bidirectional=False,
                              q_start=None, upcast=torch.float64):
    """``(out, lse)`` of (B, H, S, D) tensors; differentiable through autograd."""
    b, hq, q_len, _ = q.shape
    hkv, kv_len = k.shape[1], k.shape[2]
    rep = hq // hkv
    qf, kf, vf = (x.to(upcast) for x in (q, k, v))
    kf = kf.repeat_interleave(rep, dim=1)
    vf = vf.repeat_interleave(rep, dim=1)
    scores = torch.einsum("bhqd,bhkd->bhqk", qf, kf)
    mask = gemma4_attention_mask(
        batch_size=b, q_len=q_len, kv_len=kv_len, sliding_window=sliding_window,
        vision_block_ids=None if vision_block_ids is None else np.asarray(vision_block_ids),
        document_ids=None if document_ids is None else np.asarray(document_ids),
        q_start=q_start, allow_vision_bidirectional=allow_vision_bidirectional)
    scores = scores.masked_fill(~torch.from_numpy(np.asarray(mask)), float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    probs = torch.exp(scores - lse[..., None])
    probs = torch.where(torch.isfinite(lse)[..., None], probs, torch.zeros_like(probs))
    out = torch.einsum("bhqk,bhkd->bhqd", probs, vf).to(q.dtype)
    return out, lse.to(torch.float32)
