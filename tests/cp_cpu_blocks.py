"""Float64 CPU stand-in for the block computations of context parallelism
(test infrastructure; ``gemma4_fa4_kernels_b200.context_parallel.CudaBlocks``
is the product path).  Same contract as the CUDA blocks:

* ``fwd``: one block's output and LSE (lower-right alignment plus the causal
  shift for global layers; the exact oracle mask for local layers);
* ``bwd_acc``: the block's gradient contributions ADDED to dq / dk / dv, from
  the final output and LSE of the whole row (the flash-attention identities
  P = exp(S - LSE), dV = P^T dO, dS = P (dO V^T - rowsum(dO * O) + dLSE),
  dQ = dS K, dK = dS^T Q; ``reference.py:23-75`` differentiated), GQA summed
  over each KV head's query group;
* ``merge`` / ``cast`` / ``add_`` as in ``g4_merge_attention_partial``,
  ``g4_cast_f32_bf16`` and ``g4_add_f32``.
"""

from __future__ import annotations

import numpy as np
import torch

import oracle
from oracle.masks import gemma4_attention_mask


def _allowed(sq, sk, *, shift, window, vision_ids, document_ids):
    # the kernels' contract (g4_attn_args): every query keeps q_abs >= 0, and the
    # shift applies to global layers only
    assert sk - sq + shift >= 0, "Sq may exceed Sk only by the causal shift"
    assert shift == 0 or not window, "causal shift on a local layer"
    if not window:
        q_abs = torch.arange(sq)[:, None] + (sk - sq + shift)
        return torch.arange(sk)[None, :] <= q_abs
    m = gemma4_attention_mask(
        batch_size=1, q_len=sq, kv_len=sk, sliding_window=window,
        vision_block_ids=None if vision_ids is None else vision_ids.reshape(1, -1).numpy(),
        document_ids=None if document_ids is None else document_ids.reshape(1, -1).numpy(),
        allow_vision_bidirectional=True)
    return torch.from_numpy(np.asarray(m[0, 0]))


class CpuBlocks:
    def fwd(self, q, k, v, *, shift=0, window=0, vision_ids=None, document_ids=None):
        sq, sk = q.shape[1], k.shape[1]
        allowed = _allowed(sq, sk, shift=shift, window=window, vision_ids=vision_ids,
                           document_ids=document_ids)
        rep = q.shape[2] // k.shape[2]
        kk = k[0].repeat_interleave(rep, dim=1).transpose(0, 1)  # (H, Sk, D)
        vv = v[0].repeat_interleave(rep, dim=1).transpose(0, 1)
        s = torch.einsum("qhd,hkd->hqk", q[0], kk).masked_fill(~allowed, float("-inf"))
        lse = torch.logsumexp(s, dim=-1)  # (H, Sq)
        p = torch.where(torch.isfinite(lse)[..., None], torch.exp(s - lse[..., None]),
                        torch.zeros_like(s))
        o = torch.einsum("hqk,hkd->qhd", p, vv)
        return o[None], lse[None]

    def bwd_acc(self, q, k, v, o, lse, do, dlse, dq, dk, dv, *, shift=0, window=0,
                vision_ids=None, document_ids=None):
        sq, sk = q.shape[1], k.shape[1]
        allowed = _allowed(sq, sk, shift=shift, window=window, vision_ids=vision_ids,
                           document_ids=document_ids)
        hq, hkv = q.shape[2], k.shape[2]
        rep = hq // hkv
        kk = k[0].repeat_interleave(rep, dim=1).transpose(0, 1)
        vv = v[0].repeat_interleave(rep, dim=1).transpose(0, 1)
        s = torch.einsum("qhd,hkd->hqk", q[0], kk)
        l0 = lse[0]
        p = torch.where(allowed[None] & torch.isfinite(l0)[..., None], torch.exp(s - l0[..., None]),
                        torch.zeros_like(s))
        dout = do[0].transpose(0, 1)  # (H, Sq, D)
        delta = (do[0] * o[0]).sum(-1).transpose(0, 1)  # (H, Sq)
        if dlse is not None:
            delta = delta - torch.where(torch.isfinite(l0), dlse[0], torch.zeros_like(dlse[0]))
        dp = torch.einsum("hqd,hkd->hqk", dout, vv)
        ds = p * (dp - delta[..., None])
        dq[0] += torch.einsum("hqk,hkd->qhd", ds, kk).to(dq.dtype)
        dkh = torch.einsum("hqk,qhd->hkd", ds, q[0])
        dvh = torch.einsum("hqk,hqd->hkd", p, dout)
        dk[0] += dkh.reshape(hkv, rep, sk, -1).sum(1).transpose(0, 1).to(dk.dtype)
        dv[0] += dvh.reshape(hkv, rep, sk, -1).sum(1).transpose(0, 1).to(dv.dtype)

    def merge(self, o_acc, lse_acc, o_part, lse_part):
        m = torch.maximum(lse_acc, lse_part)
        fin = torch.isfinite(m)
        ms = torch.where(fin, m, torch.zeros_like(m))
        ea, eb = torch.exp(lse_acc - ms), torch.exp(lse_part - ms)
        ssum = ea + eb
        wa = torch.where(fin, ea / ssum, torch.ones_like(ea))
        wb = torch.where(fin, eb / ssum, torch.zeros_like(eb))
        o_acc.copy_(o_acc * wa[0].transpose(0, 1)[None, ..., None]
                    + o_part.to(o_acc.dtype) * wb[0].transpose(0, 1)[None, ..., None])
        lse_acc.copy_(torch.where(fin, ms + torch.log(ssum), m))

    def cast(self, x):
        return x.clone()

    def add_(self, dst, src):
        dst += src


def reference(q, k, v, do, *, window=0, vision_ids=None, document_ids=None, dlse=None):
    """Whole-sequence oracle: (out, lse, dq, dk, dv) in BSHD / (B,H,S)."""
    t = lambda x: x.numpy().transpose(0, 2, 1, 3)  # noqa: E731
    kw = dict(sliding_window=window or None, allow_vision_bidirectional=bool(window),
              vision_block_ids=None if vision_ids is None else vision_ids.reshape(1, -1).numpy(),
              document_ids=None if document_ids is None else document_ids.reshape(1, -1).numpy())
    o, lse = oracle.attention_fwd(t(q), t(k), t(v), **kw)
    dq, dk, dv = oracle.attention_bwd(t(q), t(k), t(v), t(do),
                                      dlse=None if dlse is None else dlse.numpy(), **kw)
    back = lambda x: torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3)))  # noqa: E731
    return back(o), torch.from_numpy(lse.astype(np.float64)), back(dq), back(dk), back(dv)
