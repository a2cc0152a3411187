"""Transformers backend: Gemma-4 text attention through the B200 kernels.

``register_gemma4_fa4_b200()`` registers an attention function and a mask
function under ``BACKEND_NAME`` in Transformers' attention and mask registries
(idempotent; a different function already registered under the name is an
error), so that a Gemma-4 model loaded with ``attn_implementation="gemma4_fa4_b200"``
runs its sliding (d256, window 1024) and full (d512, causal) attention layers
on the CUDA kernels of this package (reference: transformers_integration.py:
3500-3550 registration, 1702-2098 prepared routing, 118-189 mask plan).

The mask function returns a ``Gemma4MaskPlan``: the composed mask predicate
that Transformers built (causal, sliding overlay, packed sequences, padding)
plus its query/key geometry, unevaluated.  The attention function checks that
predicate against the kernels' own mask before it dispatches: it evaluates the
plan with Transformers' ``sdpa_mask`` on the query rows (all of them when the
mask is small, otherwise the first and last rows and every row next to a
packed-sequence boundary) and compares with ``g4_build_mask`` for the
candidate native mask (with or without documents taken from ``position_ids``).
The reference proves the same equality by parsing the pinned mask closures;
evaluation needs no pinned Transformers revision.  A mismatch, padding, or a
sliding-window cache whose keys are not the positions 0..K-1 raises
``UnsupportedB200Path`` before any launch (``allow_sdpa_fallback=True`` routes
such calls to PyTorch SDPA with the dense Transformers mask instead).

Dispatch: equal query and key lengths use the autograd path (fixed layout, or
packed segments for global layers with packed sequences); shorter query spans
against a cache (decode, chunked prefill) use the lower-right fixed layout
without autograd; a single query token takes the split-key decode kernels.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Callable

import torch

from . import b200, ops
from .errors import UnsupportedB200Path
from .model_spec import GLOBAL_ATTENTION, SLIDING_ATTENTION, AttentionLayerSpec

BACKEND_NAME = "gemma4_fa4_b200"

# Masks up to this many elements are compared in full; larger ones on sampled rows.
_FULL_CHECK_ELEMENTS = 1 << 24
_EDGE_ROWS = 64


@dataclass(frozen=True)
class Gemma4MaskPlan:
    """The mask information Transformers hands to the mask interface, kept
    unevaluated for the attention function."""

    batch_size: int
    q_length: int
    kv_length: int
    q_offset: int
    kv_offset: int
    mask_function: Callable | None
    attention_mask: torch.Tensor | None


@dataclass(frozen=True)
class Gemma4DispatchResult:
    """Attention output with the implementation path that produced it."""

    output: torch.Tensor
    lse: torch.Tensor | None
    path: str


def _as_int(value: int | torch.Tensor) -> int:
    if isinstance(value, torch.Tensor):
        if value.numel() != 1:
            raise ValueError("mask offsets must be scalars")
        return int(value.item())
    return int(value)


def gemma4_fa4_b200_mask(batch_size: int, q_length: int, kv_length: int,
                         q_offset: int | torch.Tensor = 0, kv_offset: int | torch.Tensor = 0,
                         mask_function: Callable | None = None,
                         attention_mask: torch.Tensor | None = None, **_kwargs) -> Gemma4MaskPlan:
    """Mask-interface entry: record the plan, evaluate nothing."""
    return Gemma4MaskPlan(int(batch_size), int(q_length), int(kv_length), _as_int(q_offset),
                          _as_int(kv_offset), mask_function, attention_mask)


def _spec_for_module(module: Any, query: torch.Tensor, key: torch.Tensor) -> AttentionLayerSpec:
    sliding = bool(getattr(module, "is_sliding", False))
    base = SLIDING_ATTENTION if sliding else GLOBAL_ATTENTION
    return replace(base, num_q_heads=int(query.shape[1]), num_kv_heads=int(key.shape[1]))


def _validate_semantics(module: Any, spec: AttentionLayerSpec, query: torch.Tensor, *,
                        dropout: float, scaling: float | None, sliding_window: int | None,
                        output_attentions: bool) -> None:
    if output_attentions:
        raise UnsupportedB200Path("the B200 backend does not return attention probabilities")
    if dropout:
        raise UnsupportedB200Path("attention dropout is not part of the Gemma-4 contract")
    if scaling is not None and float(scaling) != spec.softmax_scale:
        raise UnsupportedB200Path("Gemma-4 attention uses softmax scale 1.0")
    if query.shape[-1] != spec.head_dim_qk:
        raise UnsupportedB200Path(
            f"{spec.kind} layers use head dim {spec.head_dim_qk}, got {query.shape[-1]}")
    if spec.kind == "sliding_attention" and sliding_window != spec.sliding_window:
        raise UnsupportedB200Path(f"sliding layers use window {spec.sliding_window}")
    if spec.kind == "full_attention" and sliding_window is not None:
        raise UnsupportedB200Path("full attention layers take no sliding window")


def _packed_documents(position_ids: torch.Tensor | None, batch: int,
                      length: int) -> torch.Tensor | None:
    """Sequence index of every token when ``position_ids`` restart inside a row
    (Transformers' packed-sequence convention), else None."""
    if position_ids is None or position_ids.dim() != 2 or position_ids.shape[-1] != length:
        return None
    pos = position_ids.expand(batch, -1)
    starts = torch.ones_like(pos, dtype=torch.bool)
    starts[:, 1:] = pos[:, 1:] - pos[:, :-1] != 1
    docs = starts.to(torch.int32).cumsum(-1, dtype=torch.int32) - 1
    if int(docs[:, -1].max().item()) == 0:
        return None
    return docs.contiguous()


def _check_rows(q_length: int, kv_length: int, batch: int,
                documents: torch.Tensor | None) -> list[tuple[int, int]]:
    """Contiguous query-row blocks on which the two masks are compared."""
    if batch * q_length * kv_length <= _FULL_CHECK_ELEMENTS:
        return [(0, q_length)]
    rows = {(0, min(_EDGE_ROWS, q_length)), (max(0, q_length - _EDGE_ROWS), q_length)}
    if documents is not None:
        starts = torch.nonzero(documents[:, 1:] != documents[:, :-1])[:, 1] + 1
        for s in torch.unique(starts).tolist()[:256]:
            rows.add((max(0, s - 2), min(q_length, s + 2)))
    return sorted(rows)


def _transformers_rows(plan: Gemma4MaskPlan, row0: int, rows: int,
                       device: torch.device) -> torch.Tensor:
    from transformers.masking_utils import sdpa_mask

    mask = sdpa_mask(batch_size=plan.batch_size, q_length=rows, kv_length=plan.kv_length,
                     q_offset=plan.q_offset + row0, kv_offset=plan.kv_offset,
                     mask_function=plan.mask_function, attention_mask=plan.attention_mask,
                     allow_is_causal_skip=False, allow_torch_fix=False, use_vmap=False,
                     device=device)
    return mask[:, 0].to(torch.bool)


def _native_rows(plan: Gemma4MaskPlan, spec: AttentionLayerSpec, documents, row0: int,
                 rows: int, valid: int, device: torch.device) -> torch.Tensor:
    """The kernels' mask for query rows [row0, row0 + rows) against key
    positions 0..kv_length-1 (keys at or past ``valid`` are outside the cache)."""
    window = spec.sliding_window or 0
    doc_rows = None
    if documents is not None:
        doc_rows = torch.full((plan.batch_size, plan.kv_length), -1, dtype=torch.int32,
                              device=device)
        doc_rows[:, :documents.shape[1]] = documents
    dense = ops.build_mask(plan.batch_size, rows, plan.kv_length, window=window,
                           allow_vision_bidirectional=False, document_ids=doc_rows,
                           q_start=plan.q_offset + row0, device=device).to(torch.bool)
    if valid < plan.kv_length:
        dense[:, :, valid:] = False
    if documents is not None:  # a query's own document is the documents row at its position
        q_docs = documents[:, plan.q_offset + row0:plan.q_offset + row0 + rows]
        dense &= (doc_rows.unsqueeze(1) == q_docs.unsqueeze(-1))
    return dense


def _plan_matches(plan, spec, documents, valid, device) -> bool:
    for row0, row1 in _check_rows(plan.q_length, plan.kv_length, plan.batch_size, documents):
        hf = _transformers_rows(plan, row0, row1 - row0, device)
        mine = _native_rows(plan, spec, documents, row0, row1 - row0, valid, device)
        if not torch.equal(hf, mine):
            return False
    return True


def _sdpa_fallback(plan: Gemma4MaskPlan, query, key, value, spec) -> Gemma4DispatchResult:
    mask = _transformers_rows(plan, 0, plan.q_length, query.device).unsqueeze(1)
    rep = query.shape[1] // key.shape[1]
    k = key[:, :, :plan.kv_length].repeat_interleave(rep, dim=1)
    v = value[:, :, :plan.kv_length].repeat_interleave(rep, dim=1)
    out = torch.nn.functional.scaled_dot_product_attention(query, k, v, attn_mask=mask,
                                                           scale=spec.softmax_scale)
    return Gemma4DispatchResult(out.transpose(1, 2), None, "sdpa_fallback")


def gemma4_fa4_b200_prepared(module: Any, query: torch.Tensor, key: torch.Tensor,
                             value: torch.Tensor, attention_mask: Gemma4MaskPlan | None, *,
                             dropout: float = 0.0, scaling: float | None = 1.0,
                             sliding_window: int | None = None,
                             position_ids: torch.Tensor | None = None,
                             output_attentions: bool = False, allow_sdpa_fallback: bool = False,
                             **_kwargs) -> Gemma4DispatchResult:
    """Route Transformers' prepared ``(B, H, S, D)`` Q/K/V to the kernels."""
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise ValueError("Transformers attention passes (B, H, S, D) tensors")
    spec = _spec_for_module(module, query, key)
    _validate_semantics(module, spec, query, dropout=dropout, scaling=scaling,
                        sliding_window=sliding_window, output_attentions=output_attentions)
    plan = attention_mask
    if not isinstance(plan, Gemma4MaskPlan):
        raise UnsupportedB200Path(
            f"expected the {BACKEND_NAME!r} mask plan; register both entries with "
            "register_gemma4_fa4_b200()")
    batch, _, q_len, _ = query.shape
    if plan.batch_size != batch or plan.q_length != q_len or key.shape[2] < plan.kv_length:
        raise ValueError("the mask plan does not describe these tensors")

    def unsupported(reason: str) -> Gemma4DispatchResult:
        if allow_sdpa_fallback:
            return _sdpa_fallback(plan, query, key, value, spec)
        raise UnsupportedB200Path(reason)

    if plan.kv_offset != 0:
        return unsupported("keys must be the positions 0..K-1 (no rolled sliding-window cache)")
    valid = plan.q_offset + q_len  # keys a causal query row can reach
    if valid > plan.kv_length:
        return unsupported("queries extend past the key range")
    if plan.attention_mask is not None and not bool(
            plan.attention_mask[:, :valid].to(torch.bool).all().item()):
        return unsupported("padded batches are not routed to the kernels")
    documents = _packed_documents(position_ids, batch, q_len) if q_len == valid else None
    candidates = [documents, None] if documents is not None else [None]
    chosen = "none"
    for docs in candidates:
        if _plan_matches(plan, spec, docs, valid, query.device):
            chosen = docs
            break
    if isinstance(chosen, str):
        return unsupported("the Transformers mask differs from the Gemma-4 kernel mask")
    documents = chosen

    q = query.transpose(1, 2)
    k = key[:, :, :valid].transpose(1, 2)
    v = value[:, :, :valid].transpose(1, 2)
    window = spec.sliding_window or 0
    b200._validate_bshd(q, k, v, spec, label="transformers backend")
    if q_len < valid:
        if torch.is_grad_enabled() and any(t.requires_grad for t in (query, key, value)):
            return unsupported("gradients through a cache (query shorter than keys) are not routed")
        with torch.no_grad():
            out, lse = ops.attn_fwd(q, k, v, window=window)
        return Gemma4DispatchResult(out, lse, "decode" if q_len == 1 else "prefix")
    if documents is None:
        out, lse = b200._run(q, k, v, window=window)
        return Gemma4DispatchResult(out, lse, f"{spec.kind}_fixed")
    if spec.kind == "sliding_attention":
        out, lse = b200._run(q, k, v, window=window, documents=documents.contiguous())
        return Gemma4DispatchResult(out, lse, "sliding_attention_documents")
    # global layers: one packed segment per sequence of the batch rows
    bounds = [0]
    for row in range(batch):
        d = documents[row]
        cuts = (torch.nonzero(d[1:] != d[:-1]).flatten() + 1).tolist()
        bounds += [row * q_len + c for c in cuts] + [(row + 1) * q_len]
    cu = torch.tensor(bounds, dtype=torch.int32, device=query.device)
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    qp = q.reshape(batch * q_len, *q.shape[2:])
    kp = k.reshape(batch * q_len, *k.shape[2:])
    vp = v.reshape(batch * q_len, *v.shape[2:])
    out, lse = b200._run(qp, kp, vp, window=0, cu_q=cu, cu_k=cu, max_q=max(lengths),
                         max_k=max(lengths))
    return Gemma4DispatchResult(out.reshape(batch, q_len, *out.shape[1:]), lse,
                                "full_attention_packed")


def gemma4_fa4_b200_attention_forward(module: Any, query: torch.Tensor, key: torch.Tensor,
                                      value: torch.Tensor,
                                      attention_mask: Gemma4MaskPlan | None, **kwargs):
    """Transformers attention-interface entry: ``(attn_output (B, S, H, D), None)``."""
    result = gemma4_fa4_b200_prepared(module, query, key, value, attention_mask, **kwargs)
    try:
        module._gemma4_fa4_b200_last_path = result.path
    except (AttributeError, TypeError):  # pragma: no cover - frozen modules
        pass
    return result.output, None


def _registered(registry: Any, key: str):
    try:
        return registry[key]
    except (KeyError, TypeError):
        return None


def register_gemma4_fa4_b200(attention_registry: Any = None, mask_registry: Any = None) -> str:
    """Register the attention and mask entries under ``BACKEND_NAME``
    (idempotent).  The registries default to Transformers' global ones."""
    if attention_registry is None or mask_registry is None:
        try:
            from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
            from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
        except Exception as exc:  # pragma: no cover - optional dependency
            raise RuntimeError("Transformers is required for backend registration") from exc
        attention_registry = attention_registry or ALL_ATTENTION_FUNCTIONS
        mask_registry = mask_registry or ALL_MASK_ATTENTION_FUNCTIONS
    targets = ((attention_registry, gemma4_fa4_b200_attention_forward, "attention"),
               (mask_registry, gemma4_fa4_b200_mask, "mask"))
    for registry, fn, label in targets:
        existing = _registered(registry, BACKEND_NAME)
        if existing is not None and existing is not fn:
            raise RuntimeError(f"Transformers {label} backend {BACKEND_NAME!r} is already registered")
    for registry, fn, _ in targets:
        if _registered(registry, BACKEND_NAME) is None:
            registry.register(BACKEND_NAME, fn)
    return BACKEND_NAME
