"""Low-level operators: torch tensors in, C-ABI call, torch tensors out.

These functions do only what the native boundary needs (pointer/stride
marshalling, output and workspace allocation on the caller's stream, status
to exception mapping).  Contract validation that the reference performs in its
adapters lives in ``b200.py``.  Every call runs on the current CUDA
stream; nothing here synchronises the host.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .errors import UnsupportedB200Path


def _raise_for(status: int, what: str) -> None:
    if status == _lib.G4_OK:
        return
    msg = f"{what}: {_lib.last_error()}"
    if status == _lib.G4_ERR_INVALID:
        raise ValueError(msg)
    if status == _lib.G4_ERR_UNSUPPORTED:
        raise UnsupportedB200Path(msg)
    raise RuntimeError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _strides3(t: torch.Tensor, packed: bool):
    arr = (ctypes.c_int64 * 3)()
    if packed:  # (T, H, D)
        arr[0], arr[1], arr[2] = 0, t.stride(0), t.stride(1)
    else:  # (B, S, H, D)
        arr[0], arr[1], arr[2] = t.stride(0), t.stride(1), t.stride(2)
    return arr


def _meta(x: torch.Tensor | None, device) -> torch.Tensor | None:
    if x is None:
        return None
    if x.device != device:
        raise ValueError("metadata must be on the operand device")
    return x.to(torch.int32).contiguous()


def _build_args(q, k, v, o, lse, *, window, vision_ids, document_ids, cu_seqlens_q,
                cu_seqlens_k, max_seqlen_q, max_seqlen_k):
    packed = cu_seqlens_q is not None
    a = _lib.G4AttnArgs()
    a.q, a.k, a.v, a.o, a.lse = _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse)
    a.q_stride = _strides3(q, packed)
    a.k_stride = _strides3(k, packed)
    a.v_stride = _strides3(v, packed)
    a.o_stride = _strides3(o, packed)
    if packed:
        a.batch = cu_seqlens_q.numel() - 1
        a.seqlen_q, a.seqlen_k = q.shape[0], k.shape[0]
        a.cu_seqlens_q, a.cu_seqlens_k = _ptr(cu_seqlens_q), _ptr(cu_seqlens_k)
        a.max_seqlen_q, a.max_seqlen_k = int(max_seqlen_q), int(max_seqlen_k)
        a.num_q_heads, a.num_kv_heads = q.shape[1], k.shape[1]
        a.lse_stride[0], a.lse_stride[1] = 0, lse.stride(0)
    else:
        a.batch, a.seqlen_q, a.seqlen_k = q.shape[0], q.shape[1], k.shape[1]
        a.num_q_heads, a.num_kv_heads = q.shape[2], k.shape[2]
        a.lse_stride[0], a.lse_stride[1] = lse.stride(0), lse.stride(1)
    a.head_dim_qk, a.head_dim_v = q.shape[-1], v.shape[-1]
    a.window = int(window or 0)
    a.vision_ids, a.document_ids = _ptr(vision_ids), _ptr(document_ids)
    return a


# Argument blocks and workspace sizes depend only on shapes, strides, flags and
# which optional tensors are present, not on the data: a call with a known
# signature copies its cached block and writes the pointers.  (Marshalling the
# block field by field costs more host time than a short kernel.)
_SIG_CACHE: dict = {}
_SIG_CACHE_MAX = 512


def _sig(t: torch.Tensor | None):
    return None if t is None else (tuple(t.shape), t.stride())


def _cached_args(key, build, sizes):
    """(argument block, workspace sizes) of a signature: a fresh copy of the
    cached block (pointers still to be written) and the sizes `sizes(block)`
    computed once."""
    hit = _SIG_CACHE.get(key)
    if hit is None:
        a = build()
        hit = (bytes(a), sizes(a))
        if len(_SIG_CACHE) >= _SIG_CACHE_MAX:
            _SIG_CACHE.clear()
        _SIG_CACHE[key] = hit
    return _lib.G4AttnArgs.from_buffer_copy(hit[0]), hit[1]


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# The materialised-P/dS backward and the two-pass forward run band by band:
# each band's tiles fit the workspace.  The workspace is the whole problem's
# scratch when that fits this budget (the smaller of 64 GiB and a third of the
# device's memory), else the budget itself, which the library cuts into bands.
# The budget is fixed per device: querying free memory on every call costs more
# than a whole backward at the benchmark sizes.
_SCRATCH_CAP = 64 * 1024**3
_budget_cache: dict[int, int] = {}


def _scratch_budget(device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _budget_cache:
        total = torch.cuda.get_device_properties(idx).total_memory
        _budget_cache[idx] = min(_SCRATCH_CAP, total // 3)
    return _budget_cache[idx]


def _pick_workspace(full: int, small: int, force_small: bool, device,
                    budget: int | None = None) -> torch.Tensor:
    """Workspace for the fast (scratch-backed) path: the whole problem's
    scratch, or the budget when that is smaller (the library then runs bands);
    the minimum workspace of the compact path when forced or out of memory."""
    if force_small:
        return _workspace(small, device)
    size = max(min(full, _scratch_budget(device) if budget is None else int(budget)), small)
    try:
        return _workspace(size, device)
    except torch.cuda.OutOfMemoryError:
        return _workspace(small, device)


# The raw handle of the current stream without building a Stream object (a
# microsecond per call on the host); the public API where torch lacks it.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device) -> int:
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def attn_fwd(q, k, v, *, window=0, vision_ids=None, document_ids=None, cu_seqlens_q=None,
             cu_seqlens_k=None, max_seqlen_q=None, max_seqlen_k=None, out=None,
             algorithm="auto", causal_shift=0, workspace_bytes=None):
    """Forward through ``g4_attn_fwd``.  Fixed BSHD (4-D) or packed THD (3-D)
    inputs; returns ``(out, lse)`` with LSE ``(B,Hq,Sq)`` or ``(Hq,Tq)``.

    ``algorithm``: "auto" lets global d512 run the two-pass forward (in bands
    when its scratch exceeds the budget); "single" forces the single-kernel
    forward.  ``causal_shift`` (global layers) moves every query ``shift``
    positions to the right of its lower-right position; ``workspace_bytes``
    overrides the budget (tests use it to force several bands)."""
    lib = _lib.load()
    packed = cu_seqlens_q is not None
    dev = q.device
    if out is None:
        out = torch.empty(*q.shape[:-1], v.shape[-1], dtype=q.dtype, device=dev)
    if packed:
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
    else:
        lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=torch.float32, device=dev)
    vis, doc = _meta(vision_ids, dev), _meta(document_ids, dev)

    def build():
        a = _build_args(q, k, v, out, lse, window=window, vision_ids=vis, document_ids=doc,
                        cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
                        max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k)
        a.causal_shift = int(causal_shift)
        return a

    key = ("fwd", dev.index, q.dtype, _sig(q), _sig(k), _sig(v), _sig(out), _sig(lse),
           int(window or 0), vis is not None, doc is not None, _sig(cu_seqlens_q),
           _sig(cu_seqlens_k), max_seqlen_q, max_seqlen_k, int(causal_shift))
    a, (full, small) = _cached_args(
        key, build, lambda a: (lib.g4_attn_fwd_workspace_bytes(ctypes.byref(a)),
                               lib.g4_attn_fwd_min_workspace_bytes(ctypes.byref(a))))
    a.q, a.k, a.v, a.o, a.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr()
    a.vision_ids, a.document_ids = _ptr(vis), _ptr(doc)
    a.cu_seqlens_q, a.cu_seqlens_k = _ptr(cu_seqlens_q), _ptr(cu_seqlens_k)
    ws = _pick_workspace(full, small, algorithm in ("single", "recompute"), dev, workspace_bytes)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _raise_for(lib.g4_attn_fwd(ctypes.byref(a), _stream(dev)), "g4_attn_fwd")
    return out, lse


def attn_bwd(q, k, v, out, lse, dout, *, dlse=None, window=0, vision_ids=None,
             document_ids=None, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=None,
             max_seqlen_k=None, dq=None, dk=None, dv=None, algorithm="auto", causal_shift=0,
             accumulate=False, workspace_bytes=None):
    """Backward through ``g4_attn_bwd``; returns ``(dq, dk, dv)``.

    ``algorithm``: "auto" materialises P/dS (in bands when the scratch exceeds
    the budget), "recompute" always passes the minimum workspace (recompute
    kernels).  ``accumulate``: ``dq``/``dk``/``dv`` are fp32 tensors and the
    gradients are added to them (ring partial sums).  ``causal_shift`` and
    ``workspace_bytes`` as in :func:`attn_fwd`."""
    lib = _lib.load()
    packed = cu_seqlens_q is not None
    dev = q.device
    if accumulate and (dq is None or dk is None or dv is None):
        raise ValueError("accumulate=True needs fp32 dq, dk and dv to add into")
    if accumulate and any(t.dtype != torch.float32 for t in (dq, dk, dv)):
        raise ValueError("accumulated gradients must be float32")
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    vis, doc = _meta(vision_ids, dev), _meta(document_ids, dev)
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    if dlse is not None:
        dlse = dlse.to(torch.float32).contiguous()
        if dlse.shape != lse.shape:
            raise ValueError("dlse must match the LSE shape")
    if algorithm not in ("auto", "materialized", "recompute"):
        raise ValueError(f"unknown backward algorithm {algorithm!r}")

    def build():
        a = _build_args(q, k, v, out, lse, window=window, vision_ids=vis, document_ids=doc,
                        cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
                        max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k)
        a.dout = _ptr(dout)
        a.dlse = _ptr(dlse)
        a.do_stride = _strides3(dout, packed)
        a.dq, a.dk, a.dv = _ptr(dq), _ptr(dk), _ptr(dv)
        a.dq_stride = _strides3(dq, packed)
        a.dk_stride = _strides3(dk, packed)
        a.dv_stride = _strides3(dv, packed)
        a.causal_shift = int(causal_shift)
        a.grad_accumulate = 1 if accumulate else 0
        return a

    key = ("bwd", dev.index, q.dtype, dq.dtype, _sig(q), _sig(k), _sig(v), _sig(out), _sig(lse),
           _sig(dout), dlse is not None, _sig(dq), _sig(dk), _sig(dv), int(window or 0),
           vis is not None, doc is not None, _sig(cu_seqlens_q), _sig(cu_seqlens_k),
           max_seqlen_q, max_seqlen_k, int(causal_shift), bool(accumulate))
    a, (full, small) = _cached_args(
        key, build, lambda a: (lib.g4_attn_bwd_workspace_bytes(ctypes.byref(a)),
                               lib.g4_attn_bwd_min_workspace_bytes(ctypes.byref(a))))
    a.q, a.k, a.v, a.o, a.lse = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr()
    a.vision_ids, a.document_ids = _ptr(vis), _ptr(doc)
    a.cu_seqlens_q, a.cu_seqlens_k = _ptr(cu_seqlens_q), _ptr(cu_seqlens_k)
    a.dout, a.dlse = dout.data_ptr(), _ptr(dlse)
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    ws = _pick_workspace(full, small, algorithm == "recompute", dev, workspace_bytes)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _raise_for(lib.g4_attn_bwd(ctypes.byref(a), _stream(dev)), "g4_attn_bwd")
    return dq, dk, dv


def build_mask(batch, q_len, kv_len, *, window, allow_vision_bidirectional, vision_ids=None,
               document_ids=None, key_padding_mask=None, q_start=None, device):
    """Dense ``(B, Q, K)`` uint8 mask from ``g4_build_mask``."""
    lib = _lib.load()
    out = torch.empty(batch, q_len, kv_len, dtype=torch.uint8, device=device)
    vis, doc = _meta(vision_ids, device), _meta(document_ids, device)
    pad = None if key_padding_mask is None else key_padding_mask.to(torch.uint8).contiguous()
    rc = lib.g4_build_mask(_ptr(out), batch, q_len, kv_len, -1 if q_start is None else int(q_start),
                           int(window or 0),
                           int(bool(allow_vision_bidirectional)), _ptr(vis), _ptr(doc), _ptr(pad),
                           _stream(device))
    _raise_for(rc, "g4_build_mask")
    return out


def _rows_view(t: torch.Tensor):
    """(tokens, heads, d) strides of a (1, S, H, D) or (T, H, D) tensor."""
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError("merges take one sequence (batch 1) or a packed tensor")
        return t.shape[1], t.shape[2], t.shape[3], t.stride(1), t.stride(2)
    return t.shape[0], t.shape[1], t.shape[2], t.stride(0), t.stride(1)


def _lse_view(lse: torch.Tensor):
    """(head, token) strides of a (1, H, S) or (H, T) LSE."""
    if lse.dim() == 3:
        return lse.stride(1), lse.stride(2)
    return lse.stride(0), lse.stride(1)


def merge_partial(o_acc, lse_acc, o_part, lse_part) -> None:
    """In place: fp32 ``o_acc`` / ``lse_acc`` <- the exact softmax merge with a
    block's bf16 output ``o_part`` and LSE ``lse_part``
    (``g4_merge_attention_partial``)."""
    if o_acc.dtype != torch.float32 or lse_acc.dtype != torch.float32:
        raise ValueError("o_acc and lse_acc must be float32")
    if o_part.dtype != torch.bfloat16 or lse_part.dtype != torch.float32:
        raise ValueError("o_part must be bfloat16 and lse_part float32")
    lib = _lib.load()
    tok, heads, d, ts, hs = _rows_view(o_acc)
    ptok, pheads, pd, pts, phs = _rows_view(o_part)
    if (tok, heads, d) != (ptok, pheads, pd) or o_acc.stride(-1) != 1 or o_part.stride(-1) != 1:
        raise ValueError("o_acc and o_part must have the same rows, heads and unit feature stride")
    a = _lib.G4MergeArgs()
    a.o_acc, a.lse_acc = o_acc.data_ptr(), lse_acc.data_ptr()
    a.o_part, a.lse_part = o_part.data_ptr(), lse_part.data_ptr()
    a.o_acc_stride[:] = [ts, hs]
    a.o_part_stride[:] = [pts, phs]
    a.lse_acc_stride[:] = list(_lse_view(lse_acc))
    a.lse_part_stride[:] = list(_lse_view(lse_part))
    a.tokens, a.heads, a.head_dim = tok, heads, d
    _raise_for(lib.g4_merge_attention_partial(ctypes.byref(a), _stream(o_acc.device)),
               "g4_merge_attention_partial")


def cast_f32_bf16(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 copy of a contiguous fp32 ``(1, S, H, D)`` / ``(T, H, D)`` tensor
    (``g4_cast_f32_bf16``)."""
    if src.dtype != torch.float32 or not src.is_contiguous():
        raise ValueError("src must be a contiguous float32 tensor")
    out = torch.empty(src.shape, dtype=torch.bfloat16, device=src.device) if out is None else out
    tok, heads, d, _, _ = _rows_view(src)
    _, _, _, ts, hs = _rows_view(out)
    lib = _lib.load()
    _raise_for(lib.g4_cast_f32_bf16(src.data_ptr(), out.data_ptr(), tok, heads, d, ts, hs,
                                    _stream(src.device)), "g4_cast_f32_bf16")
    return out


def add_f32_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """In place ``dst += src`` for contiguous float32 tensors of equal size
    (``g4_add_f32``)."""
    if dst.dtype != torch.float32 or src.dtype != torch.float32:
        raise ValueError("dst and src must be float32")
    if not (dst.is_contiguous() and src.is_contiguous()) or dst.numel() != src.numel():
        raise ValueError("dst and src must be contiguous with equal sizes")
    lib = _lib.load()
    _raise_for(lib.g4_add_f32(dst.data_ptr(), src.data_ptr(), dst.numel(), _stream(dst.device)),
               "g4_add_f32")
    return dst
