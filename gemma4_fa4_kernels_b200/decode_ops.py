"""Single-token static-cache decode layer ops for Gemma-4 (B=1, Q=1).

The opaque operators of the reference's compiled decode path
(src/gemma4_fa4/h100_torch_ops.py:479-880, registered at :1007-1017): one
decoding step of one attention layer -- projections, Q/K RMS norms, rotary
embedding, the KV-cache mutation, attention over the active cache and the
output projection -- as ``torch.library`` custom ops that declare the caches
they mutate, with fake implementations for tracing.

* global layer (d512, 32Q/4KV, K and V from the same projection):
  writes the new K (RoPE(KNorm(Z))) and V (VNorm(Z)) at slot ``cache_length``
  of (1, 4, capacity, 512) caches, advances ``cache_length`` by one and attends
  over the first ``cache_length`` slots (h100_torch_ops.py:805-880);
* local layer (d256, 32Q/16KV, window 1024): below position 1024 writes slot
  ``cache_length`` of (1, 16, 1024, 256) caches; from position 1024 on it rolls
  the caches left by one slot and writes the last slot, as the sliding-window
  cache layer does (h100_torch_ops.py:692-803); ``cache_length`` is read only.

The attention runs on the split-key decode kernels of this package through
``ops.attn_fwd`` on (1, L, H, D) views of the caches (no copy); the reference
pads the query to the cache length below position 1024 and otherwise calls
its packed forward, both of which equal this single-row lower-right result.
Projections are plain cuBLAS BF16 GEMMs (``torch.nn.functional.linear``); the
Q/K norms, the rotary embedding and the value norm run in the fused
``g4_prep_fwd`` kernel (global layers: K and V from one read of Z).
"""

from __future__ import annotations

import torch

from . import ops
from .errors import UnsupportedB200Path
from .prep import prep_fwd

HIDDEN_SIZE = 5376
LOCAL_GEOMETRY = (32, 16, 256)   # query heads, KV heads, head dim
GLOBAL_GEOMETRY = (32, 4, 512)
LOCAL_WINDOW = 1024              # local cache slots (= sliding window)
MAX_POSITION = 262144

GLOBAL_STATIC_CACHE_DECODE_OP_NAME = "gemma4_fa4_b200::global_static_cache_decode_fwd"
LOCAL_STATIC_CACHE_DECODE_OP_NAME = "gemma4_fa4_b200::local_static_cache_decode_fwd"


# ------------------------------------------------------------------------------------
# admission (reference h100_torch_ops.py:479-690, with the B200 capability)
# ------------------------------------------------------------------------------------
def _common_checks(label, hidden_states, cos, sin, position_ids, cache_k, cache_v, cache_length,
                   weights, rot_dim):
    explicit = (hidden_states, cos, sin, position_ids, cache_k, cache_v, cache_length, *weights)
    if hidden_states.shape != (1, 1, HIDDEN_SIZE):
        raise UnsupportedB200Path(f"{label} decode requires B1, Q1 and hidden size {HIDDEN_SIZE}")
    if hidden_states.device.type != "cuda" or any(t.device != hidden_states.device for t in explicit):
        raise UnsupportedB200Path(f"{label} decode tensors must share one CUDA device")
    cap = torch.cuda.get_device_capability(hidden_states.device)
    if cap != (10, 0):
        raise UnsupportedB200Path(f"{label} decode requires compute capability 10.0, found {cap}")
    if any(t.dtype != torch.bfloat16 for t in (hidden_states, cos, sin, cache_k, cache_v, *weights)):
        raise ValueError(f"{label} decode activations, caches and weights must be BF16")
    if cos.shape != (1, 1, rot_dim) or sin.shape != (1, 1, rot_dim):
        raise ValueError(f"{label} decode rotary tensors must be (1, 1, {rot_dim})")
    if position_ids.shape != (1, 1) or position_ids.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"{label} decode position_ids must be INT32/INT64 (1, 1)")
    if cache_length.ndim != 0 or cache_length.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"{label} decode cache length must be a scalar integer tensor")
    if any(t.requires_grad for t in (hidden_states, cos, sin, cache_k, cache_v)):
        raise UnsupportedB200Path(f"{label} decode rejects requires_grad activations or caches")
    if any(not t.is_contiguous() for t in explicit):
        raise ValueError(f"{label} decode inputs must be contiguous")
    if len({t.untyped_storage().data_ptr() for t in explicit}) != len(explicit):
        raise ValueError(f"{label} decode arguments must use distinct storage")


def _check_weights(label, weights, shapes):
    if len(weights) != len(shapes):
        raise AssertionError(f"{label} decode weight schema is inconsistent")
    for w, shape in zip(weights, shapes, strict=True):
        if w.shape != shape:
            raise ValueError(f"{label} decode weight of shape {tuple(w.shape)} conflicts with "
                             f"the locked layer ({shape})")


def _validate_global(hidden_states, cos, sin, position_ids, cache_k, cache_v, cache_length,
                     weights) -> int:
    hq, hkv, d = GLOBAL_GEOMETRY
    _common_checks("global static-cache", hidden_states, cos, sin, position_ids, cache_k, cache_v,
                   cache_length, weights, d)
    if cache_k.ndim != 4 or cache_k.shape[:2] != (1, hkv) or cache_k.shape[-1] != d:
        raise ValueError(f"global static cache must be (1, {hkv}, capacity, {d})")
    if cache_v.shape != cache_k.shape:
        raise ValueError("global K/V caches must have equal geometry")
    capacity = cache_k.shape[2]
    length = int(cache_length.item())
    if not 1 <= length < MAX_POSITION:
        raise UnsupportedB200Path("global static-cache decode requires a nonempty in-range prefix")
    if capacity > MAX_POSITION or length + 1 >= capacity:
        raise UnsupportedB200Path("global static-cache decode requires spare unwritten capacity")
    if int(position_ids.item()) != length:
        raise UnsupportedB200Path("the decode position must equal the active prefix length")
    _check_weights("global static-cache", weights,
                   ((hq * d, HIDDEN_SIZE), (hkv * d, HIDDEN_SIZE), (HIDDEN_SIZE, hq * d), (d,), (d,)))
    return length


def _validate_local(hidden_states, cos, sin, position_ids, cache_k, cache_v, cache_length,
                    weights) -> int:
    hq, hkv, d = LOCAL_GEOMETRY
    _common_checks("local sliding-cache", hidden_states, cos, sin, position_ids, cache_k, cache_v,
                   cache_length, weights, d)
    if cache_k.shape != (1, hkv, LOCAL_WINDOW, d) or cache_v.shape != cache_k.shape:
        raise ValueError(f"local sliding caches must be (1, {hkv}, {LOCAL_WINDOW}, {d})")
    position = int(position_ids.item())
    if not 1 <= position < MAX_POSITION:
        raise UnsupportedB200Path("local sliding-cache decode requires a nonempty in-range prefix")
    if int(cache_length.item()) != min(position, LOCAL_WINDOW):
        raise UnsupportedB200Path("the sliding cache length conflicts with the absolute position")
    _check_weights("local sliding-cache", weights,
                   ((hq * d, HIDDEN_SIZE), (hkv * d, HIDDEN_SIZE), (hkv * d, HIDDEN_SIZE),
                    (HIDDEN_SIZE, hq * d), (d,), (d,)))
    return position


# ------------------------------------------------------------------------------------
# implementations
# ------------------------------------------------------------------------------------
T = torch.Tensor


def _global_impl(hidden_states: T, cos: T, sin: T, position_ids: T, cache_k: T, cache_v: T,
                 cache_length: T, q_proj_weight: T, k_proj_weight: T, o_proj_weight: T,
                 q_norm_weight: T, k_norm_weight: T) -> tuple[T, T]:
    weights = (q_proj_weight, k_proj_weight, o_proj_weight, q_norm_weight, k_norm_weight)
    length = _validate_global(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                              cache_length, weights)
    hq, hkv, d = GLOBAL_GEOMETRY
    lin = torch.nn.functional.linear
    q, _ = prep_fwd(lin(hidden_states, q_proj_weight).view(1, 1, hq, d), q_norm_weight, cos, sin,
                    d)
    k, v = prep_fwd(lin(hidden_states, k_proj_weight).view(1, 1, hkv, d), k_norm_weight, cos, sin,
                    d, want_plain=True)
    slot = torch.arange(1, device=cache_k.device) + cache_length
    cache_k.index_copy_(2, slot, k.transpose(1, 2))
    cache_v.index_copy_(2, slot, v.transpose(1, 2))
    cache_length.add_(1)
    active = length + 1
    attn, lse = ops.attn_fwd(q, cache_k[:, :, :active].transpose(1, 2),
                             cache_v[:, :, :active].transpose(1, 2), window=0)
    out = lin(attn.reshape(1, 1, hq * d), o_proj_weight)
    return out, lse


def _local_impl(hidden_states: T, cos: T, sin: T, position_ids: T, cache_k: T, cache_v: T,
                cache_length: T, q_proj_weight: T, k_proj_weight: T, v_proj_weight: T,
                o_proj_weight: T, q_norm_weight: T, k_norm_weight: T) -> tuple[T, T]:
    weights = (q_proj_weight, k_proj_weight, v_proj_weight, o_proj_weight, q_norm_weight,
               k_norm_weight)
    position = _validate_local(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                               cache_length, weights)
    hq, hkv, d = LOCAL_GEOMETRY
    lin = torch.nn.functional.linear
    q, _ = prep_fwd(lin(hidden_states, q_proj_weight).view(1, 1, hq, d), q_norm_weight, cos, sin,
                    d)
    k, _ = prep_fwd(lin(hidden_states, k_proj_weight).view(1, 1, hkv, d), k_norm_weight, cos, sin,
                    d)
    _, v = prep_fwd(lin(hidden_states, v_proj_weight).view(1, 1, hkv, d), None, None, None, 0,
                    want_rot=False, want_plain=True)
    k, v = k.transpose(1, 2), v.transpose(1, 2)
    if position < LOCAL_WINDOW:
        slot = torch.arange(1, dtype=cache_length.dtype, device=cache_k.device) + cache_length
        cache_k.index_copy_(2, slot, k)
        cache_v.index_copy_(2, slot, v)
        active = position + 1
    else:  # the window is full: shift every slot left by one, append at the end
        cache_k.copy_(torch.cat((cache_k[:, :, 1:], k), dim=2))
        cache_v.copy_(torch.cat((cache_v[:, :, 1:], v), dim=2))
        active = LOCAL_WINDOW
    attn, lse = ops.attn_fwd(q, cache_k[:, :, :active].transpose(1, 2),
                             cache_v[:, :, :active].transpose(1, 2), window=LOCAL_WINDOW)
    out = lin(attn.reshape(1, 1, hq * d), o_proj_weight)
    return out, lse


def _fake(hidden_states, *_args):
    out = torch.empty((hidden_states.shape[0], hidden_states.shape[1], HIDDEN_SIZE),
                      dtype=hidden_states.dtype, device=hidden_states.device)
    lse = torch.empty((hidden_states.shape[0], GLOBAL_GEOMETRY[0], hidden_states.shape[1]),
                      dtype=torch.float32, device=hidden_states.device)
    return out, lse


global_static_cache_decode_op = torch.library.custom_op(
    GLOBAL_STATIC_CACHE_DECODE_OP_NAME, mutates_args={"cache_k", "cache_v", "cache_length"})(
    _global_impl)
torch.library.register_fake(GLOBAL_STATIC_CACHE_DECODE_OP_NAME)(_fake)

local_static_cache_decode_op = torch.library.custom_op(
    LOCAL_STATIC_CACHE_DECODE_OP_NAME, mutates_args={"cache_k", "cache_v"})(_local_impl)
torch.library.register_fake(LOCAL_STATIC_CACHE_DECODE_OP_NAME)(_fake)


def _check_call_boundary(hidden_states, cos, sin) -> None:
    """Reject autograd before the custom op disables grad mode for its body."""
    if torch.is_grad_enabled():
        raise UnsupportedB200Path("static-cache decode ops require inference / no-grad mode")
    names = [n for n, t in zip(("hidden_states", "cos", "sin"), (hidden_states, cos, sin))
             if t.requires_grad]
    if names:
        raise UnsupportedB200Path("static-cache decode ops reject requires_grad activations: "
                                  + ", ".join(names))


def global_static_cache_decode_fwd(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                                   cache_length, q_proj_weight, k_proj_weight, o_proj_weight,
                                   q_norm_weight, k_norm_weight):
    """One global-layer decode step; mutates ``cache_k``, ``cache_v`` and
    ``cache_length``.  Returns ``(out (1, 1, 5376) BF16, lse (1, 32, 1) FP32)``."""
    _check_call_boundary(hidden_states, cos, sin)
    return global_static_cache_decode_op(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                                         cache_length, q_proj_weight, k_proj_weight,
                                         o_proj_weight, q_norm_weight, k_norm_weight)


def local_static_cache_decode_fwd(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                                  cache_length, q_proj_weight, k_proj_weight, v_proj_weight,
                                  o_proj_weight, q_norm_weight, k_norm_weight):
    """One local-layer decode step; mutates ``cache_k`` and ``cache_v``.
    Returns ``(out (1, 1, 5376) BF16, lse (1, 32, 1) FP32)``."""
    _check_call_boundary(hidden_states, cos, sin)
    return local_static_cache_decode_op(hidden_states, cos, sin, position_ids, cache_k, cache_v,
                                        cache_length, q_proj_weight, k_proj_weight, v_proj_weight,
                                        o_proj_weight, q_norm_weight, k_norm_weight)
