"""Contract adapters for the B200 (sm_100a) kernels.

Same operator surface as the reference's H100 adapters
(``src/gemma4_fa4/h100.py``): the fixed-BSHD and packed-THD local-d256 and
global-d512 entry points with the same names, keyword arguments, return values
``(out, lse)``, exception types and admission order (every check runs before
any launch).  Differences, all on the permissive side:

* the envelope is the model maximum (B >= 1, sequence lengths up to 262144)
  instead of the reference's H100 evidence limits (B = 1, S <= 1025 local /
  2048 global-with-backward);
* the global d512 output is produced by one kernel, not two V256 slab
  launches, so there is no cross-slab LSE check to fail;
* backward of every adapter supports a gradient on the returned LSE;
* head counts may be a divisor of the model's (one GPU's share of a head
  partition), keeping the GQA ratio.

Compute runs in ``libgemma4_b200.so``; there is no CPU or library fallback.
"""

from __future__ import annotations

import torch

from . import ops
from .errors import GlobalBackwardBudgetExceeded, UnsupportedB200Path
from .model_spec import GEMMA4_31B, GLOBAL_ATTENTION, SLIDING_ATTENTION, AttentionLayerSpec

_MODEL_MAX_SEQLEN = GEMMA4_31B.max_position_embeddings
_GLOBAL_BACKWARD_RESERVE_BYTES = 2 * 1024**3

__all__ = [
    "fa4_local_text_forward",
    "fa4_local_forward",
    "fa4_local_varlen_forward",
    "fa4_global_text_forward",
    "fa4_global_forward_only",
    "fa4_global_varlen_forward",
    "fa4_global_varlen_forward_only",
]


# ------------------------------------------------------------------------------------
# validation helpers (mirroring h100.py:123-367, 634-747, 920-1145)
# ------------------------------------------------------------------------------------
def _is_fake_tensor(tensor: torch.Tensor) -> bool:
    try:
        from torch._subclasses.fake_tensor import FakeTensor
    except ImportError:  # pragma: no cover
        return False
    return isinstance(tensor, FakeTensor)


def _require_sm100(device: torch.device) -> None:
    if device.type != "cuda":
        raise UnsupportedB200Path("B200 inputs must be CUDA tensors")
    capability = torch.cuda.get_device_capability(device)
    if capability != (10, 0):
        raise UnsupportedB200Path(f"B200 kernels require compute capability 10.0, found {capability}")


def _has_proven_nonoverlap(tensor: torch.Tensor) -> bool:
    """Mixed-radix proof that a positive-stride layout does not overlap: with
    non-trivial modes sorted by stride, every stride must exceed the span of
    all smaller modes (accepts gapped static-cache prefix views)."""
    overlap = torch._debug_has_internal_overlap(tensor)
    if overlap == 0:
        return True
    if overlap == 1:
        return False
    span = 0
    for stride, size in sorted((st, sz) for sz, st in zip(tensor.shape, tensor.stride()) if sz > 1):
        if stride <= span:
            return False
        span += (size - 1) * stride
    return True


def _validate_layout(tensor: torch.Tensor, *, name: str) -> None:
    if tensor.stride(-1) != 1:
        raise ValueError(f"{name} must have unit last-dimension stride")
    if any(stride <= 0 for stride in tensor.stride()):
        raise ValueError(f"{name} must use positive, non-broadcast strides")
    if any(stride % 8 for stride in tensor.stride()[:-1]):
        raise ValueError(f"{name} outer strides must be 16-byte aligned for BF16")
    if not _has_proven_nonoverlap(tensor):
        raise ValueError(f"{name} must use a non-overlapping layout")


def _check_operands(q, k, v, *, rank: int, label: str) -> bool:
    """Common operand checks; returns True when all inputs are fake tensors."""
    if any(t.ndim != rank for t in (q, k, v)):
        shape = "B/S/H/D" if rank == 4 else "T/H/D"
        raise ValueError(f"{label} q, k, and v must be rank-{rank} {shape} tensors")
    if not (q.device == k.device == v.device):
        raise ValueError(f"{label} q, k, and v must be on one device")
    if any(t.dtype != torch.bfloat16 for t in (q, k, v)):
        raise ValueError(f"{label} accepts BF16 q, k, and v only")
    for name, tensor in zip(("q", "k", "v"), (q, k, v)):
        _validate_layout(tensor, name=f"{label} {name}".strip())
    fake = [_is_fake_tensor(t) for t in (q, k, v)]
    if any(fake) and not all(fake):
        raise ValueError("q, k, and v must all be real tensors or all be fake tensors")
    if not all(fake):
        if any(t.data_ptr() % 16 for t in (q, k, v)):
            raise ValueError("q, k, and v base pointers must be 16-byte aligned")
        if k.untyped_storage().data_ptr() == v.untyped_storage().data_ptr():
            raise ValueError("K and V must be distinct, non-aliasing prepared operands")
    return all(fake)


def _check_heads(spec: AttentionLayerSpec, model: AttentionLayerSpec) -> bool:
    """Head counts must be the model's or one GPU's share of a head partition
    over 2, 4 or 8 GPUs: query heads split evenly, each share keeping exactly
    the KV heads its query heads read."""
    if spec.num_q_heads <= 0 or spec.num_kv_heads <= 0:
        return False
    if model.num_q_heads % spec.num_q_heads:
        return False
    if model.num_q_heads // spec.num_q_heads not in {1, 2, 4, 8}:
        return False
    return spec.num_kv_heads == max(1, spec.num_q_heads // model.qhead_per_kvhead)


def _local_contract(spec: AttentionLayerSpec) -> bool:
    return (spec.kind == "sliding_attention" and spec.head_dim_qk == 256 and spec.head_dim_v == 256
            and spec.softmax_scale == 1.0 and spec.sliding_window == 1024 and spec.is_causal
            and _check_heads(spec, SLIDING_ATTENTION))


def _global_contract(spec: AttentionLayerSpec) -> bool:
    return (spec.kind == "full_attention" and spec.head_dim_qk == 512 and spec.head_dim_v == 512
            and spec.softmax_scale == 1.0 and spec.sliding_window is None and spec.is_causal
            and _check_heads(spec, GLOBAL_ATTENTION))


def _validate_bshd(q, k, v, spec, *, require_sm100=True, label="") -> bool:
    fake = _check_operands(q, k, v, rank=4, label=label)
    batch, seqlen, q_heads, q_dim = q.shape
    if batch <= 0 or seqlen <= 0:
        raise ValueError("batch and sequence length must be positive")
    kv_len = k.shape[1]
    if (q_heads, q_dim) != (spec.num_q_heads, spec.head_dim_qk):
        raise ValueError("q shape does not match the attention spec")
    if k.shape != (batch, kv_len, spec.num_kv_heads, spec.head_dim_qk) or \
            v.shape != (batch, kv_len, spec.num_kv_heads, spec.head_dim_v):
        raise ValueError("k/v shapes do not match the attention spec")
    if spec.qhead_per_kvhead not in {1, 2, 4, 8}:
        raise ValueError("the validated GQA ratios are 1, 2, 4, and 8")
    if require_sm100 and not fake:
        _require_sm100(q.device)
    return fake


def _validate_local_bshd(q, k, v, spec, *, require_sm100=True) -> bool:
    fake = _validate_bshd(q, k, v, spec, require_sm100=False)
    if q.shape[1] != k.shape[1]:
        raise ValueError("fixed local attention requires equal Q and K lengths")
    if q.shape[1] > _MODEL_MAX_SEQLEN:
        raise UnsupportedB200Path(f"local attention covers 1 <= S <= {_MODEL_MAX_SEQLEN}")
    if not _local_contract(spec):
        raise UnsupportedB200Path("only the locked local d256 attention contract is enabled")
    if require_sm100 and not fake:
        _require_sm100(q.device)
    return fake


def _validate_global_bshd(q, k, v, spec, *, require_sm100=True) -> bool:
    fake = _validate_bshd(q, k, v, spec, require_sm100=False)
    if q.shape[1] != k.shape[1]:
        raise ValueError("global text attention requires equal Q and K lengths")
    if q.shape[1] > _MODEL_MAX_SEQLEN:
        raise UnsupportedB200Path(f"global attention covers 1 <= S <= {_MODEL_MAX_SEQLEN}")
    if not _global_contract(spec):
        raise UnsupportedB200Path("only the locked global d512 text-forward contract is enabled")
    if require_sm100 and not fake:
        _require_sm100(q.device)
    return fake


def _normalize_int32_metadata(values: torch.Tensor, *, name: str) -> torch.Tensor:
    if values.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"{name} must use INT32 or INT64 values")
    if values.requires_grad:
        raise ValueError(f"{name} must not require gradients")
    if values.dtype == torch.int64 and not _is_fake_tensor(values):
        lo, hi = torch.aminmax(values)
        info = torch.iinfo(torch.int32)
        if lo.item() < info.min or hi.item() > info.max:
            raise ValueError(f"INT64 {name} values must fit exactly in INT32")
    return values.to(dtype=torch.int32).contiguous()


def _prepare_fixed_metadata(values, q, *, name):
    if values is None:
        return None
    expected = tuple(q.shape[:2])
    if tuple(values.shape) != expected:
        raise ValueError(f"{name} must have shape {expected}, got {tuple(values.shape)}")
    if values.device != q.device:
        raise ValueError(f"{name} must be on the same device as q, k, and v")
    return _normalize_int32_metadata(values, name=name)


def _prepare_packed_metadata(values, k, *, name):
    if values is None:
        return None
    if tuple(values.shape) != (k.shape[0],):
        raise ValueError(f"{name} must have shape ({k.shape[0]},)")
    if values.device != k.device:
        raise ValueError(f"{name} must share the q/k/v device")
    if _is_fake_tensor(values) != _is_fake_tensor(k):
        raise ValueError(f"{name} and packed q/k/v must share real/fake tensor mode")
    return _normalize_int32_metadata(values, name=name)


def _validate_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, spec,
                     *, contract, label, require_sm100=True):
    fake = _check_operands(q, k, v, rank=3, label=label)
    if q.shape[0] <= 0 or k.shape[0] <= 0:
        raise ValueError("packed Q and K totals must be positive")
    if tuple(q.shape[1:]) != (spec.num_q_heads, spec.head_dim_qk):
        raise ValueError("packed q shape does not match the attention spec")
    if tuple(k.shape[1:]) != (spec.num_kv_heads, spec.head_dim_qk):
        raise ValueError("packed k shape does not match the attention spec")
    if tuple(v.shape) != (k.shape[0], spec.num_kv_heads, spec.head_dim_v):
        raise ValueError("packed v shape does not match the attention spec")
    if not contract(spec):
        raise UnsupportedB200Path(f"only the locked {label} varlen contract is enabled")
    if any(isinstance(x, bool) or not isinstance(x, int) for x in (max_seqlen_q, max_seqlen_k)):
        raise TypeError("max_seqlen_q and max_seqlen_k must be Python integers")
    if not (1 <= max_seqlen_q <= max_seqlen_k <= _MODEL_MAX_SEQLEN):
        raise UnsupportedB200Path(
            f"packed maxima must satisfy 1 <= max Sq <= max Sk <= {_MODEL_MAX_SEQLEN}")
    cum = (cu_seqlens_q, cu_seqlens_k)
    if any(t.ndim != 1 or t.numel() < 2 for t in cum):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be rank-1 B+1 tensors")
    if cu_seqlens_q.shape != cu_seqlens_k.shape:
        raise ValueError("cu_seqlens_q and cu_seqlens_k must have the same batch count")
    if any(t.device != q.device for t in cum):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must share the q/k/v device")
    if any(t.dtype != torch.int32 for t in cum):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must use INT32")
    if any(not t.is_contiguous() for t in cum):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must be contiguous")
    fake_cum = [_is_fake_tensor(t) for t in cum]
    if any(fake_cum) and not all(fake_cum):
        raise ValueError("cu_seqlens_q and cu_seqlens_k must share real/fake tensor mode")
    if all(fake_cum) != fake:
        raise ValueError("packed q/k/v and cumulative arrays must share real/fake tensor mode")
    if fake:
        return None, None, True
    # Host read of the cumulative arrays, as the reference does (h100.py:351-352):
    # admission must know the true segment lengths before any launch.
    qv = [int(x) for x in cu_seqlens_q.detach().cpu().tolist()]
    kv = [int(x) for x in cu_seqlens_k.detach().cpu().tolist()]
    if qv[0] != 0 or kv[0] != 0:
        raise ValueError("cumulative arrays must start at zero")
    if qv[-1] != q.shape[0] or kv[-1] != k.shape[0]:
        raise ValueError("cumulative arrays must end at the packed Q/K totals")
    ql = [e - s for s, e in zip(qv[:-1], qv[1:])]
    kl = [e - s for s, e in zip(kv[:-1], kv[1:])]
    if any(x < 0 for x in (*ql, *kl)):
        raise ValueError("cumulative arrays must be nondecreasing")
    if any(a > b for a, b in zip(ql, kl)):
        raise UnsupportedB200Path("each packed sequence requires Sq <= Sk")
    if max(ql) != max_seqlen_q or max(kl) != max_seqlen_k:
        raise ValueError("max_seqlen_q/max_seqlen_k must equal the cumulative maxima")
    if require_sm100:
        _require_sm100(q.device)
    return ql, kl, False


def _backward_budget(free_bytes: int) -> int:
    return min(free_bytes * 4 // 5, max(0, free_bytes - _GLOBAL_BACKWARD_RESERVE_BYTES))


def _preflight_backward(q, k, v, *, packed_batch: int | None = None) -> None:
    """Fail closed before the forward when the backward would not fit: the
    gradients (same sizes as q, k, v) plus the kernel workspace (two fp32 rows
    per query head and token, tile lists) against the guarded free-HBM budget."""
    if _is_fake_tensor(q) or q.device.type != "cuda":
        return
    tokens = q.shape[0] if packed_batch is not None else q.shape[0] * q.shape[1]
    heads = q.shape[-2]
    workspace = 8 * heads * tokens + 16 * (tokens // 128 + (packed_batch or 0) + 2) + 4096
    grads = sum(t.numel() * t.element_size() for t in (q, k, v))
    required = grads + workspace
    free, _total = torch.cuda.mem_get_info(q.device)
    budget = _backward_budget(free)
    if required > budget:
        raise GlobalBackwardBudgetExceeded(
            f"backward needs about {required} additional bytes, above the guarded budget of "
            f"{budget} bytes ({free} bytes currently free)")


def _preflight_forward_outputs(q) -> None:
    if _is_fake_tensor(q) or q.device.type != "cuda":
        return
    required = q.numel() * q.element_size() + (q.numel() // q.shape[-1]) * 4
    free, _total = torch.cuda.mem_get_info(q.device)
    if required > free * 8 // 10:
        raise UnsupportedB200Path(
            f"forward outputs require about {required} bytes, above 80% of the {free} free bytes")


def _fake_outputs(q, v, packed):
    out = torch.empty(*q.shape[:-1], v.shape[-1], dtype=q.dtype, device=q.device)
    if packed:
        lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    else:
        lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=torch.float32, device=q.device)
    return out, lse


# ------------------------------------------------------------------------------------
# autograd: one Function for every layout / mask combination
# ------------------------------------------------------------------------------------
class _AttentionFunction(torch.autograd.Function):
    """Forward through g4_attn_fwd, backward through g4_attn_bwd (dO and dLSE)."""

    @staticmethod
    def forward(ctx, q, k, v, window, vision, documents, cu_q, cu_k, max_q, max_k):
        kw = dict(window=window, vision_ids=vision, document_ids=documents, cu_seqlens_q=cu_q,
                  cu_seqlens_k=cu_k, max_seqlen_q=max_q, max_seqlen_k=max_k)
        out, lse = ops.attn_fwd(q, k, v, **kw)
        ctx.save_for_backward(q, k, v, out, lse, vision, documents, cu_q, cu_k)
        ctx.window, ctx.max_q, ctx.max_k = window, max_q, max_k
        ctx.set_materialize_grads(False)
        return out, lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, k, v, out, lse, vision, documents, cu_q, cu_k = ctx.saved_tensors
        if dout is None and dlse is None:
            return (None,) * 10
        if dout is None:
            dout = torch.zeros_like(out)
        dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, dout, dlse=dlse, window=ctx.window,
                                  vision_ids=vision, document_ids=documents, cu_seqlens_q=cu_q,
                                  cu_seqlens_k=cu_k, max_seqlen_q=ctx.max_q,
                                  max_seqlen_k=ctx.max_k)
        return dq, dk, dv, None, None, None, None, None, None, None


def _run(q, k, v, *, window, vision=None, documents=None, cu_q=None, cu_k=None, max_q=None,
         max_k=None, allow_grad=True):
    needs_grad = torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v))
    if needs_grad and allow_grad:
        return _AttentionFunction.apply(q, k, v, window, vision, documents, cu_q, cu_k, max_q,
                                        max_k)
    with torch.no_grad():
        return ops.attn_fwd(q, k, v, window=window, vision_ids=vision, document_ids=documents,
                            cu_seqlens_q=cu_q, cu_seqlens_k=cu_k, max_seqlen_q=max_q,
                            max_seqlen_k=max_k)


# ------------------------------------------------------------------------------------
# public adapters
# ------------------------------------------------------------------------------------
def fa4_local_text_forward(q, k, v, *, spec: AttentionLayerSpec = SLIDING_ATTENTION):
    """Fixed-length Gemma local text attention (window 1024, causal).

    ``(B, S, H, D)`` BF16 inputs with unit D stride; returns ``(out, lse)`` with
    LSE FP32 ``(B, Hq, S)``.  Autograd supplies dQ/dK/dV (h100.py:750-778).
    """
    if _validate_local_bshd(q, k, v, spec):
        return _fake_outputs(q, v, packed=False)
    return _run(q, k, v, window=spec.sliding_window)


def fa4_local_forward(q, k, v, *, vision_block_ids=None, spec: AttentionLayerSpec = SLIDING_ATTENTION):
    """Fixed-length local attention with the exact vision overlay
    (h100.py:781-815): keys in the query's non-negative vision block are
    visible in both directions, still bounded by the strict left window."""
    if vision_block_ids is None:
        return fa4_local_text_forward(q, k, v, spec=spec)
    fake = _validate_local_bshd(q, k, v, spec)
    ids = _prepare_fixed_metadata(vision_block_ids, q, name="vision_block_ids")
    if fake:
        return _fake_outputs(q, v, packed=False)
    return _run(q, k, v, window=spec.sliding_window, vision=ids)


def fa4_local_varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, *, max_seqlen_q, max_seqlen_k,
                             vision_block_ids=None, document_ids=None,
                             spec: AttentionLayerSpec = SLIDING_ATTENTION):
    """Packed local self-attention (h100.py:818-911): each Q segment is the
    lower-right suffix of its K segment; vision/document ids follow the packed
    K stream (defaults -1 / 0).  One launch covers every segment, with or
    without metadata; there is no per-segment loop or host-built schedule."""
    _, _, fake = _validate_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                  spec, contract=_local_contract, label="local d256")
    vis = _prepare_packed_metadata(vision_block_ids, k, name="vision_block_ids")
    docs = _prepare_packed_metadata(document_ids, k, name="document_ids")
    if fake:
        return _fake_outputs(q, v, packed=True)
    return _run(q, k, v, window=spec.sliding_window, vision=vis, documents=docs, cu_q=cu_seqlens_q,
                cu_k=cu_seqlens_k, max_q=max_seqlen_q, max_k=max_seqlen_k)


def fa4_global_text_forward(q, k, v, *, spec: AttentionLayerSpec = GLOBAL_ATTENTION):
    """Fixed-length global causal d512 attention with autograd
    (h100.py:1320-1394).  One launch produces all 512 output columns; the
    backward honours a gradient on LSE and materialises a missing dO as zeros.
    The backward's memory is checked before the forward runs."""
    fake = _validate_global_bshd(q, k, v, spec)
    if fake:
        return _fake_outputs(q, v, packed=False)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        _preflight_backward(q, k, v)
    else:
        _preflight_forward_outputs(q)
    return _run(q, k, v, window=0)


def fa4_global_forward_only(q, k, v, *, spec: AttentionLayerSpec = GLOBAL_ATTENTION):
    """No-grad global d512 forward for rectangular lower-right shapes
    ``1 <= Sq <= Sk <= 262144`` (h100.py:995-1036)."""
    fake = _validate_bshd(q, k, v, spec, require_sm100=False, label="global forward-only")
    if not (1 <= q.shape[1] <= k.shape[1] <= _MODEL_MAX_SEQLEN):
        raise UnsupportedB200Path("global forward-only requires B>=1 and 1 <= Sq <= Sk <= 262144")
    if not _global_contract(spec):
        raise UnsupportedB200Path("only the locked global d512 contract is enabled")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise UnsupportedB200Path(
            "global forward-only cannot participate in autograd; use fa4_global_text_forward "
            "or packed fa4_global_varlen_forward")
    if fake:
        return _fake_outputs(q, v, packed=False)
    _require_sm100(q.device)
    _preflight_forward_outputs(q)
    return _run(q, k, v, window=0, allow_grad=False)


def fa4_global_varlen_forward_only(q, k, v, cu_seqlens_q, cu_seqlens_k, *, max_seqlen_q,
                                   max_seqlen_k, spec: AttentionLayerSpec = GLOBAL_ATTENTION):
    """Packed lower-right global d512 forward without autograd (h100.py:1193-1225)."""
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise UnsupportedB200Path(
            "global packed forward-only cannot participate in autograd; use "
            "fa4_global_varlen_forward")
    _, _, fake = _validate_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                  spec, contract=_global_contract, label="global d512")
    if fake:
        return _fake_outputs(q, v, packed=True)
    _preflight_forward_outputs(q)
    return _run(q, k, v, window=0, cu_q=cu_seqlens_q, cu_k=cu_seqlens_k, max_q=max_seqlen_q,
                max_k=max_seqlen_k, allow_grad=False)


def fa4_global_varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, *, max_seqlen_q, max_seqlen_k,
                              spec: AttentionLayerSpec = GLOBAL_ATTENTION):
    """Packed global d512 forward with one coordinated backward
    (h100.py:1228-1317); segments with no queries give exact-zero K/V grads."""
    _, _, fake = _validate_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                                  spec, contract=_global_contract, label="global d512")
    if fake:
        return _fake_outputs(q, v, packed=True)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        _preflight_backward(q, k, v, packed_batch=cu_seqlens_q.numel() - 1)
    else:
        _preflight_forward_outputs(q)
    return _run(q, k, v, window=0, cu_q=cu_seqlens_q, cu_k=cu_seqlens_k, max_q=max_seqlen_q,
                max_k=max_seqlen_k)
