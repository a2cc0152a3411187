"""Context parallelism: one sequence split across GPUs (one process per GPU).

Global (causal) layers use **ring attention with a zig-zag split**.  The
sequence is cut into 2N chunks; rank r holds chunks r and 2N-1-r (one early,
one late), so every rank does the same causal work.  K/V of each rank travel
round the ring over N steps by NCCL send/recv; at step t rank r holds the K/V
of rank s = r - t and attends its own queries to them:

* t = 0: its two diagonal blocks (causal, lower-right aligned);
* s < r: both of its query chunks against chunk s (every key visible);
* s > r: its late query chunk against both held chunks (every key visible).

Every step is 2C^2 query-key pairs on every rank (C = chunk length).  A block
whose keys all precede its queries runs the ordinary kernels with a causal
shift of Sq (the mask then admits every key).  The forward merges each block's
partial output into an fp32 running output with the exact log-sum-exp
combination (``g4_merge_attention_partial``).  The backward uses the final
output and LSE, so each block's dQ / dK / dV are exact partial sums.  They are
accumulated in fp32 by the kernels themselves (``grad_accumulate``): dQ stays
on the rank, and dK / dV partials travel with K/V and reach their owner after
the N-th hop.  Communication runs on NCCL's stream and overlaps the next
block's kernels; K/V for step t+1 are requested before step t computes.

Sliding-window layers need only a halo: each rank holds one contiguous chunk
and receives the last W - 1 keys (and their metadata) of its predecessor; the
backward returns the halo's key gradients, which the predecessor adds to its
own (``g4_add_f32``).

No reference counterpart: the reference runs long global contexts on one GPU
(``src/gemma4_fa4/h100.py:713-747``).  The block computations are injectable
(``blocks=``) so that the ring and halo logic can be checked on CPU ranks
(gloo) against the float64 oracle; the default uses this package's kernels.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .errors import UnsupportedB200Path


class CudaBlocks:
    """Block computations on this GPU's kernels (the product path)."""

    def fwd(self, q, k, v, *, shift=0, window=0, vision_ids=None, document_ids=None):
        return ops.attn_fwd(q, k, v, window=window, causal_shift=shift, vision_ids=vision_ids,
                            document_ids=document_ids)

    def bwd_acc(self, q, k, v, o, lse, do, dlse, dq, dk, dv, *, shift=0, window=0,
                vision_ids=None, document_ids=None):
        ops.attn_bwd(q, k, v, o, lse, do, dlse=dlse, window=window, causal_shift=shift,
                     vision_ids=vision_ids, document_ids=document_ids, dq=dq, dk=dk, dv=dv,
                     accumulate=True)

    def merge(self, o_acc, lse_acc, o_part, lse_part):
        ops.merge_partial(o_acc, lse_acc, o_part, lse_part)

    def cast(self, x):
        return ops.cast_f32_bf16(x)

    def add_(self, dst, src):
        ops.add_f32_(dst, src)


# ------------------------------------------------------------------------------------
# sharding helpers
# ------------------------------------------------------------------------------------
def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """Rank ``rank``'s zig-zag shard: chunks r and 2N-1-r of ``2N`` equal chunks
    along ``dim``, concatenated (a new contiguous tensor)."""
    n = x.shape[dim]
    if n % (2 * world):
        raise ValueError(f"sequence length {n} is not divisible by 2 x {world} ranks")
    chunks = x.chunk(2 * world, dim=dim)
    return torch.cat((chunks[rank], chunks[2 * world - 1 - rank]), dim=dim).contiguous()


def zigzag_unshard(parts, dim: int = 1) -> torch.Tensor:
    """Inverse of :func:`zigzag_shard` given every rank's shard, in rank order."""
    world = len(parts)
    chunks = [None] * (2 * world)
    for r, p in enumerate(parts):
        a, b = p.chunk(2, dim=dim)
        chunks[r], chunks[2 * world - 1 - r] = a, b
    return torch.cat(chunks, dim=dim)


def _group_info(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _peer(group, rank):
    return dist.get_global_rank(group, rank) if group is not None else rank


def _exchange(send, recv, *, to, frm, group):
    """Post sends of ``send`` to group rank ``to`` and receives into ``recv``
    from ``frm`` (asynchronous; returns the requests)."""
    p2p = [dist.P2POp(dist.isend, t, _peer(group, to), group=group) for t in send if t is not None]
    p2p += [dist.P2POp(dist.irecv, t, _peer(group, frm), group=group) for t in recv if t is not None]
    return dist.batch_isend_irecv(p2p) if p2p else []


def _wait(reqs):
    for r in reqs:
        r.wait()


def _ring_blocks(t, s, rank, c):
    """(query rows, held key rows, causal shift) of every block at ring step t."""
    if t == 0:
        return [(slice(0, c), slice(0, c), 0), (slice(c, 2 * c), slice(0, 2 * c), 0)]
    if s < rank:
        return [(slice(0, 2 * c), slice(0, c), 2 * c)]
    return [(slice(c, 2 * c), slice(0, 2 * c), c)]


# ------------------------------------------------------------------------------------
# global layers: ring attention
# ------------------------------------------------------------------------------------
def ring_global_forward(q, k, v, *, group=None, blocks=None):
    """Forward of causal attention over a zig-zag-sharded sequence.

    ``q`` (1, 2C, Hq, D), ``k``/``v`` (1, 2C, Hkv, D): this rank's shard
    (chunks r and 2N-1-r).  Returns this rank's rows of the full sequence's
    output (bf16, like q) and LSE ``(1, Hq, 2C)`` (fp32, natural log)."""
    blocks = blocks or CudaBlocks()
    world, rank = _group_info(group)
    c = q.shape[1] // 2
    if q.shape[1] != 2 * c or k.shape[1] != 2 * c:
        raise ValueError("a zig-zag shard holds two equal chunks")
    o_acc = torch.zeros(q.shape[:-1] + (v.shape[-1],), dtype=torch.float32, device=q.device)
    lse_acc = torch.full((1, q.shape[2], 2 * c), float("-inf"), dtype=torch.float32,
                         device=q.device)
    kv, spare = [k, v], [torch.empty_like(k), torch.empty_like(v)]
    for t in range(world):
        s = (rank - t) % world
        reqs = (_exchange(kv, spare, to=(rank + 1) % world, frm=(rank - 1) % world, group=group)
                if t < world - 1 else [])
        for qr, kr, shift in _ring_blocks(t, s, rank, c):
            o, lse = blocks.fwd(q[:, qr], kv[0][:, kr], kv[1][:, kr], shift=shift)
            blocks.merge(o_acc[:, qr], lse_acc[:, :, qr], o, lse)
        _wait(reqs)
        if t < world - 1:
            kv, spare = spare, kv
    return blocks.cast(o_acc), lse_acc


def ring_global_backward(q, k, v, out, lse, dout, dlse=None, *, group=None, blocks=None):
    """Gradients (dq, dk, dv) of :func:`ring_global_forward` for this rank's
    shard; ``out``/``lse`` are the forward's final results."""
    blocks = blocks or CudaBlocks()
    world, rank = _group_info(group)
    c = q.shape[1] // 2
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    acc = [torch.zeros(k.shape, dtype=torch.float32, device=q.device),
           torch.zeros(v.shape, dtype=torch.float32, device=q.device)]
    acc_spare = [torch.empty_like(acc[0]), torch.empty_like(acc[1])]
    kv, spare = [k, v], [torch.empty_like(k), torch.empty_like(v)]
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    for t in range(world):
        s = (rank - t) % world
        kv_reqs = _exchange(kv, spare, to=nxt, frm=prv, group=group) if t < world - 1 else []
        for qr, kr, shift in _ring_blocks(t, s, rank, c):
            blocks.bwd_acc(q[:, qr], kv[0][:, kr], kv[1][:, kr], out[:, qr], lse[:, :, qr],
                           dout[:, qr], None if dlse is None else dlse[:, :, qr],
                           dq[:, qr], acc[0][:, kr], acc[1][:, kr], shift=shift)
        # the held set's accumulated dK/dV moves on with it; after the last
        # step the set arriving here is this rank's own, complete
        acc_reqs = _exchange(acc, acc_spare, to=nxt, frm=prv, group=group) if world > 1 else []
        _wait(kv_reqs)
        _wait(acc_reqs)
        if t < world - 1:
            kv, spare = spare, kv
        if world > 1:
            acc, acc_spare = acc_spare, acc
    return blocks.cast(dq), blocks.cast(acc[0]), blocks.cast(acc[1])


class _RingGlobal(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, group, blocks):
        ctx.set_materialize_grads(False)
        out, lse = ring_global_forward(q, k, v, group=group, blocks=blocks)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.group, ctx.blocks = group, blocks
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, k, v, out, lse = ctx.saved_tensors
        if dout is None:
            dout = torch.zeros_like(out)
        dq, dk, dv = ring_global_backward(q, k, v, out, lse, dout, dlse, group=ctx.group,
                                          blocks=ctx.blocks)
        return dq, dk, dv, None, None


def ring_global_attention(q, k, v, *, group=None, blocks=None):
    """Autograd entry: causal global attention of a zig-zag-sharded sequence
    (see :func:`ring_global_forward`); returns this rank's ``(out, lse)``."""
    return _RingGlobal.apply(q, k, v, group, blocks or CudaBlocks())


# ------------------------------------------------------------------------------------
# sliding-window layers: halo exchange
# ------------------------------------------------------------------------------------
def _halo_len(window, c):
    h = window - 1
    if c < h:
        raise UnsupportedB200Path(f"halo exchange needs chunks of at least W-1 = {h} tokens")
    return h


def _check_local_meta(vision_ids, document_ids, rank, world, c):
    """Metadata covers the whole sequence (S,) on every rank.  A vision span that
    reaches past this rank's chunk would need keys of the next rank."""
    if vision_ids is None:
        return
    vis = vision_ids.reshape(-1)
    doc = None if document_ids is None else document_ids.reshape(-1)
    if vis.numel() != world * c:
        raise ValueError("vision ids must cover the whole sequence")
    for b in range(1, world):  # the boundary between rank b-1 and b
        x, y = b * c - 1, b * c
        same = vis[x] >= 0 and vis[x] == vis[y] and (doc is None or doc[x] == doc[y])
        if bool(same):
            raise UnsupportedB200Path("a vision span crosses a context-parallel shard boundary; "
                                      "align the shards to image boundaries")
        if rank == b - 1 and bool(vis[x] >= 0):
            later = vis[y:] == vis[x]
            if doc is not None:
                later &= doc[y:] == doc[x]
            if bool(later.any()):
                raise UnsupportedB200Path("a vision id repeats on a later shard")


def _meta_ext(meta, rank, c, h):
    if meta is None:
        return None
    flat = meta.reshape(-1)
    lo = rank * c - (h if rank > 0 else 0)
    return flat[lo:(rank + 1) * c].reshape(1, -1).contiguous()


def halo_local_forward(q, k, v, *, window=1024, vision_ids=None, document_ids=None, group=None,
                       blocks=None):
    """Forward of sliding-window attention over contiguous shards (rank r holds
    tokens [rC, (r+1)C)): receives the predecessor's last W-1 keys.  Metadata
    (``vision_ids``/``document_ids``, shape (1, S) or (S,)) covers the whole
    sequence.  Returns this rank's ``(out, lse)``."""
    blocks = blocks or CudaBlocks()
    world, rank = _group_info(group)
    c = q.shape[1]
    h = _halo_len(window, c)
    _check_local_meta(vision_ids, document_ids, rank, world, c)
    k_ext, v_ext = _halo_kv(k, v, h, rank, world, group)
    return blocks.fwd(q, k_ext, v_ext, window=window,
                      vision_ids=_meta_ext(vision_ids, rank, c, h),
                      document_ids=_meta_ext(document_ids, rank, c, h))


def _halo_kv(k, v, h, rank, world, group):
    send = [k[:, -h:].contiguous(), v[:, -h:].contiguous()] if rank < world - 1 else [None, None]
    recv = ([torch.empty((1, h) + k.shape[2:], dtype=k.dtype, device=k.device),
             torch.empty((1, h) + v.shape[2:], dtype=v.dtype, device=v.device)]
            if rank > 0 else [None, None])
    _wait(_exchange(send, recv, to=rank + 1, frm=rank - 1, group=group))
    if rank == 0:
        return k, v
    return torch.cat((recv[0], k), dim=1), torch.cat((recv[1], v), dim=1)


def halo_local_backward(q, k, v, out, lse, dout, dlse=None, *, window=1024, vision_ids=None,
                        document_ids=None, group=None, blocks=None):
    """Gradients of :func:`halo_local_forward`; the halo's key gradients go
    back to the predecessor, which adds them to its own."""
    blocks = blocks or CudaBlocks()
    world, rank = _group_info(group)
    c = q.shape[1]
    h = _halo_len(window, c)
    k_ext, v_ext = _halo_kv(k, v, h, rank, world, group)
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    dk = torch.zeros(k_ext.shape, dtype=torch.float32, device=q.device)
    dv = torch.zeros(v_ext.shape, dtype=torch.float32, device=q.device)
    blocks.bwd_acc(q, k_ext, v_ext, out, lse, dout, dlse, dq, dk, dv, window=window,
                   vision_ids=_meta_ext(vision_ids, rank, c, h),
                   document_ids=_meta_ext(document_ids, rank, c, h))
    off = h if rank > 0 else 0
    send = [dk[:, :h].contiguous(), dv[:, :h].contiguous()] if rank > 0 else [None, None]
    recv = ([torch.empty((1, h) + dk.shape[2:], dtype=torch.float32, device=q.device),
             torch.empty((1, h) + dv.shape[2:], dtype=torch.float32, device=q.device)]
            if rank < world - 1 else [None, None])
    _wait(_exchange(send, recv, to=rank - 1, frm=rank + 1, group=group))
    # this rank's own keys (batch 1: slices along the sequence stay contiguous)
    dk_own, dv_own = dk[:, off:], dv[:, off:]
    if rank < world - 1:  # the successor's contribution to this rank's last W-1 keys
        blocks.add_(dk_own[:, -h:], recv[0])
        blocks.add_(dv_own[:, -h:], recv[1])
    return blocks.cast(dq), blocks.cast(dk_own), blocks.cast(dv_own)
