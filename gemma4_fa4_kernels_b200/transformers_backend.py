"""Transformers backend: Gemma-4 attention through the B200 kernels.

``register_gemma4_fa4_b200()`` registers an attention function and a mask
function under ``BACKEND_NAME`` in Transformers' attention and mask registries
(idempotent; a different function already registered under the name is an
error), so that a Gemma-4 model loaded with ``attn_implementation="gemma4_fa4_b200"``
runs its sliding (d256, window 1024) and full (d512, causal) attention layers
on the CUDA kernels of this package (reference: transformers_integration.py:
3500-3550 registration, 1702-2098 prepared routing, 1250-1449 packing of
padded batches, 118-189 and 543-647 mask plan and its proof).

The mask function returns a ``Gemma4MaskPlan``: the composed mask predicate
that Transformers built (causal, sliding overlay, the image overlay of
multimodal inputs, packed sequences, padding) plus its query/key geometry,
unevaluated.  Before any launch the attention function proves that predicate
equal to the kernels' own mask on EVERY (query, key) element: it evaluates the
plan with Transformers' ``sdpa_mask`` in row chunks on the device and compares
them with ``g4_build_mask`` for the candidate native mask (documents from
``position_ids`` or none; images from a ``vision_block_ids`` keyword, as the
reference's Transformers patch passes them, or from the plan itself: two
consecutive tokens of one image are the only pairs a sliding query may see
ahead of itself, so the plan's (t, t+1) entries give the image groups).  The
reference proves the equality by parsing the pinned mask closures; evaluation
needs no pinned Transformers revision.  A mismatch, padding that is not one
contiguous run per row, padding together with a cache, or a sliding-window
cache whose keys are not the positions 0..K-1 raises ``UnsupportedB200Path``
before any launch.  There is no SDPA or eager fallback.

Dispatch: equal query and key lengths use the autograd path: fixed layout, or
packed segments for padded batches (valid tokens gathered, outputs scattered
back, padded query rows zero) and for global layers with packed sequences;
shorter query spans against a cache (decode, chunked prefill) use the
lower-right fixed layout without autograd; a single query token takes the
split-key decode kernels.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Callable

import torch

from . import b200, ops
from .errors import UnsupportedB200Path
from .model_spec import GLOBAL_ATTENTION, SLIDING_ATTENTION, AttentionLayerSpec

BACKEND_NAME = "gemma4_fa4_b200"

# Mask elements compared per chunk of query rows (the whole mask is compared).
_CHECK_CHUNK_ELEMENTS = 1 << 26


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


def _valid_runs(pad: torch.Tensor) -> list[tuple[int, int]]:
    """Per batch row the one contiguous run of valid (unpadded) tokens."""
    runs = []
    for row in pad.to(torch.bool).cpu():
        idx = torch.nonzero(row).flatten()
        if idx.numel() == 0:
            raise UnsupportedB200Path("a batch row without any valid token")
        a, b = int(idx[0]), int(idx[-1]) + 1
        if b - a != idx.numel():
            raise UnsupportedB200Path("padding must leave one contiguous run of tokens per row")
        runs.append((a, b))
    return runs


def _vision_from_plan(plan: Gemma4MaskPlan, valid: int, device) -> torch.Tensor | None:
    """Image groups read off the plan: a sliding query sees a later key only
    inside its own image, so (t, t+1) allowed marks t and t+1 as one image.
    Returns (B, valid) int32 ids (-1 for text) or None when no pair is linked."""
    if plan.mask_function is None or plan.q_length < 2:
        return None
    t0 = plan.q_offset
    n = plan.q_length - 1
    b = torch.arange(plan.batch_size, device=device).view(-1, 1, 1, 1)
    h = torch.zeros(1, device=device, dtype=torch.long).view(1, 1, 1, 1)
    q = (torch.arange(n, device=device) + t0).view(1, 1, -1, 1)
    link = plan.mask_function(b, h, q, q + 1)
    link = torch.as_tensor(link, device=device).to(torch.bool).expand(plan.batch_size, 1, n, 1)
    link = link[:, 0, :, 0]
    if plan.attention_mask is not None:
        pad = plan.attention_mask.to(torch.bool)
        link = link & pad[:, t0:t0 + n] & pad[:, t0 + 1:t0 + n + 1]
    if not bool(link.any()):
        return None
    member = torch.zeros(plan.batch_size, valid, dtype=torch.bool, device=device)
    member[:, t0:t0 + n] |= link
    member[:, t0 + 1:t0 + n + 1] |= link
    start = torch.zeros_like(member)
    start[:, t0:t0 + n] = link
    start[:, t0 + 1:t0 + n] &= ~link[:, :-1]  # a run starts where the previous link is off
    ids = start.to(torch.int32).cumsum(-1, dtype=torch.int32) - 1
    return torch.where(member, ids, torch.full_like(ids, -1)).contiguous()


def _transformers_rows(plan: Gemma4MaskPlan, row0: int, rows: int,
                       device: torch.device) -> torch.Tensor:
    from transformers.masking_utils import sdpa_mask

    mask = sdpa_mask(batch_size=plan.batch_size, q_length=rows, kv_length=plan.kv_length,
                     q_offset=plan.q_offset + row0, kv_offset=plan.kv_offset,
                     mask_function=plan.mask_function, attention_mask=plan.attention_mask,
                     allow_is_causal_skip=False, allow_torch_fix=False, use_vmap=False,
                     device=device)
    return mask[:, 0].to(torch.bool)


def _pad_to(meta: torch.Tensor | None, batch: int, length: int, fill: int, device):
    if meta is None:
        return None
    out = torch.full((batch, length), fill, dtype=torch.int32, device=device)
    out[:, :meta.shape[1]] = meta
    return out


def _plan_matches(plan, spec, documents, vision, pad, valid, device) -> bool:
    """Every element of the Transformers mask equals the kernels' mask for
    query rows holding a valid token (padded query rows are not attention
    rows), keys beyond ``valid`` being outside the cache."""
    window = spec.sliding_window or 0
    doc_k = _pad_to(documents, plan.batch_size, plan.kv_length, -1, device)
    vis_k = _pad_to(vision, plan.batch_size, plan.kv_length, -1, device)
    key_pad = None
    if pad is not None:
        key_pad = torch.zeros(plan.batch_size, plan.kv_length, dtype=torch.bool, device=device)
        key_pad[:, :valid] = pad
    step = max(1, _CHECK_CHUNK_ELEMENTS // max(1, plan.batch_size * plan.kv_length))
    for row0 in range(0, plan.q_length, step):
        rows = min(step, plan.q_length - row0)
        hf = _transformers_rows(plan, row0, rows, device)
        mine = ops.build_mask(plan.batch_size, rows, plan.kv_length, window=window,
                              allow_vision_bidirectional=window > 0, vision_ids=vis_k,
                              document_ids=doc_k, key_padding_mask=key_pad,
                              q_start=plan.q_offset + row0, device=device).to(torch.bool)
        if valid < plan.kv_length:
            mine[:, :, valid:] = False
        if pad is not None:  # compare valid query rows only
            qv = pad[:, plan.q_offset + row0:plan.q_offset + row0 + rows].unsqueeze(-1)
            hf, mine = hf & qv, mine & qv
        if not torch.equal(hf, mine):
            return False
    return True


def _segments(runs, documents, q_len):
    """Packed segment bounds (flattened token index) of every valid run, split
    at document boundaries when ``documents`` is given."""
    bounds = [0]
    total = 0
    for row, (a, b) in enumerate(runs):
        cuts = []
        if documents is not None:
            d = documents[row, a:b]
            cuts = (torch.nonzero(d[1:] != d[:-1]).flatten() + 1).tolist()
        bounds += [total + c for c in cuts] + [total + b - a]
        total += b - a
    return bounds


def _packed_call(q, k, v, runs, *, window, documents, vision, split_documents):
    """Gather the valid runs into the packed layout, run the varlen kernels
    (autograd), scatter the outputs back; padded query rows get zeros."""
    batch, s = q.shape[0], q.shape[1]
    dev = q.device
    idx = torch.cat([torch.arange(r * s + a, r * s + b, device=dev) for r, (a, b) in
                     enumerate(runs)])
    flat = lambda t: t.reshape(batch * s, *t.shape[2:]).index_select(0, idx)  # noqa: E731
    qp, kp, vp = flat(q), flat(k), flat(v)
    if split_documents:
        bounds = _segments(runs, documents, s)
    else:
        bounds = _segments(runs, None, s)
    cu = torch.tensor(bounds, dtype=torch.int32, device=dev)
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    meta = lambda m: None if m is None else m.reshape(-1).index_select(0, idx).contiguous()  # noqa
    docs_p = None if split_documents else meta(documents)
    out, lse = b200._run(qp, kp, vp, window=window, vision=meta(vision), documents=docs_p,
                         cu_q=cu, cu_k=cu, max_q=max(lengths), max_k=max(lengths))
    full = out.new_zeros(batch * s, *out.shape[1:]).index_copy(0, idx, out)
    return full.reshape(batch, s, *out.shape[1:]), lse


def gemma4_fa4_b200_prepared(module: Any, query: torch.Tensor, key: torch.Tensor,
                             value: torch.Tensor, attention_mask: Gemma4MaskPlan | None, *,
                             dropout: float = 0.0, scaling: float | None = 1.0,
                             sliding_window: int | None = None,
                             position_ids: torch.Tensor | None = None,
                             output_attentions: bool = False,
                             vision_block_ids: torch.Tensor | None = None,
                             **_kwargs) -> Gemma4DispatchResult:
    """Route Transformers' prepared ``(B, H, S, D)`` Q/K/V to the kernels.
    ``vision_block_ids`` (B, S) optionally names each token's image (-1 text)."""
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
    dev = query.device
    if plan.batch_size != batch or plan.q_length != q_len or key.shape[2] < plan.kv_length:
        raise ValueError("the mask plan does not describe these tensors")
    if plan.kv_offset != 0:
        raise UnsupportedB200Path("keys must be the positions 0..K-1 (no rolled sliding-window "
                                  "cache)")
    valid = plan.q_offset + q_len  # keys a causal query row can reach
    if valid > plan.kv_length:
        raise UnsupportedB200Path("queries extend past the key range")
    pad = None
    if plan.attention_mask is not None:
        pad = plan.attention_mask[:, :valid].to(torch.bool)
        if bool(pad.all().item()):
            pad = None
    runs = None
    if pad is not None:
        if q_len != valid:
            raise UnsupportedB200Path("padded batches are routed for prefill only (no cache)")
        runs = _valid_runs(pad)
    prefill = q_len == valid
    documents = _packed_documents(position_ids, batch, q_len) if prefill else None
    sliding = spec.kind == "sliding_attention"
    vision = None
    if sliding:
        if vision_block_ids is not None:
            vision = vision_block_ids.to(device=dev, dtype=torch.int32)[:, :valid].contiguous()
        else:
            vision = _vision_from_plan(plan, valid, dev)
    chosen = "none"
    for docs in ([documents, None] if documents is not None else [None]):
        if _plan_matches(plan, spec, docs, vision, pad, valid, dev):
            chosen = docs
            break
    if isinstance(chosen, str):
        raise UnsupportedB200Path("the Transformers mask differs from the Gemma-4 kernel mask")
    documents = chosen

    q = query.transpose(1, 2)
    k = key[:, :, :valid].transpose(1, 2)
    v = value[:, :, :valid].transpose(1, 2)
    window = spec.sliding_window or 0
    b200._validate_bshd(q, k, v, spec, label="transformers backend")
    if not prefill:
        if torch.is_grad_enabled() and any(t.requires_grad for t in (query, key, value)):
            raise UnsupportedB200Path("gradients through a cache (query shorter than keys) are "
                                      "not routed")
        with torch.no_grad():
            out, lse = ops.attn_fwd(q, k, v, window=window, vision_ids=vision)
        return Gemma4DispatchResult(out, lse, "decode" if q_len == 1 else "prefix")
    if runs is not None:  # padded batch: the valid runs as packed segments
        out, lse = _packed_call(q, k, v, runs, window=window, documents=documents,
                                vision=vision, split_documents=not sliding)
        return Gemma4DispatchResult(out, lse, f"{spec.kind}_padded")
    if documents is None:
        out, lse = b200._run(q, k, v, window=window, vision=vision)
        suffix = "_vision" if vision is not None else "_fixed"
        return Gemma4DispatchResult(out, lse, spec.kind + suffix)
    if sliding:
        out, lse = b200._run(q, k, v, window=window, vision=vision,
                             documents=documents.contiguous())
        return Gemma4DispatchResult(out, lse, "sliding_attention_documents")
    # global layers: one packed segment per sequence of the batch rows
    out, lse = _packed_call(q, k, v, [(0, q_len)] * batch, window=0, documents=documents,
                            vision=None, split_documents=True)
    return Gemma4DispatchResult(out, lse, "full_attention_packed")


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
