"""Opaque ``torch.library`` operators for ``torch.compile``: the prepared
attention forwards and the whole inference layers of Gemma-4
(``src/gemma4_fa4/h100_torch_ops.py:26-29``, impls :136-476, registration
:992-1003).

* ``gemma4_fa4_b200::local_fwd`` / ``global_fwd`` -- prepared BHSD Q/K/V
  (B = 1, one sequence: ``position_ids`` = arange(S), packed ids all zero)
  to ``(out (1, S, Hq, D) BSHD, lse (1, Hq, S))``;
* ``gemma4_fa4_b200::local_layer_fwd`` / ``global_layer_fwd`` -- hidden
  states ``(1, S, 5376)`` to ``(out (1, S, 5376), lse (1, 32, S))``: q/k(/v)
  projections, the Q/K norms and rotary embedding, the value norm, the
  attention, the output projection.  Global layers read K and V from one
  projection source (K = RoPE(KNorm(Z)), V = VNorm(Z)).

B200 path: projections and the output projection are cuBLAS BF16 GEMMs
(``torch.nn.functional.linear``); the norm + rotary preparation runs in the
fused ``g4_prep_fwd`` kernel (one launch per operand, both K and V from one
read of Z on global layers) straight into the BSHD layout the attention
kernels read, so the layer needs no transpose or copy; the attention runs in
``g4_attn_fwd``.  The reference caps S at 1024 (its H100 route); these ops
accept any 1 <= S <= 262144.  All ops are inference-only, reject autograd,
and have fake implementations for tracing.
"""

from __future__ import annotations

import torch

from . import ops
from .errors import UnsupportedB200Path
from .prep import prep_fwd

LOCAL_OP_NAME = "gemma4_fa4_b200::local_fwd"
GLOBAL_OP_NAME = "gemma4_fa4_b200::global_fwd"
LOCAL_LAYER_OP_NAME = "gemma4_fa4_b200::local_layer_fwd"
GLOBAL_LAYER_OP_NAME = "gemma4_fa4_b200::global_layer_fwd"

HIDDEN_SIZE = 5376
LOCAL_GEOMETRY = (32, 16, 256)   # query heads, KV heads, head dim
GLOBAL_GEOMETRY = (32, 4, 512)
LOCAL_WINDOW = 1024
MAX_SEQLEN = 262144

T = torch.Tensor


# ------------------------------------------------------------------------------------
# admission (reference h100_torch_ops.py:39-134 and :196-300, B200 capability)
# ------------------------------------------------------------------------------------
def _check_positions(position_ids: T, packed_sequence_ids: T, seqlen: int, device, label) -> None:
    for name, t in (("position_ids", position_ids), ("packed_sequence_ids", packed_sequence_ids)):
        if t.ndim != 2 or t.shape != (1, seqlen):
            raise ValueError(f"{label} {name} must have shape (1, S)")
        if t.device != device:
            raise ValueError(f"{label} {name} must share the operand device")
        if t.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"{label} {name} must use INT32 or INT64")
    expected = torch.arange(seqlen, device=device, dtype=position_ids.dtype).unsqueeze(0)
    if not torch.equal(position_ids, expected):
        raise UnsupportedB200Path(f"{label} position_ids must equal zero-based arange(S)")
    boundaries = torch.nn.functional.pad(torch.diff(position_ids, dim=-1) != 1, (1, 0), value=False)
    if not torch.equal(packed_sequence_ids.to(torch.int64), boundaries.to(torch.int64).cumsum(-1)):
        raise UnsupportedB200Path(f"{label} packed_sequence_ids must be derived exactly from "
                                  "position_ids")


def _check_device(tensors, label) -> None:
    dev = tensors[0].device
    if dev.type != "cuda" or any(t.device != dev for t in tensors):
        raise UnsupportedB200Path(f"{label} tensors must be CUDA tensors on one device")
    cap = torch.cuda.get_device_capability(dev)
    if cap != (10, 0):
        raise UnsupportedB200Path(f"{label} requires compute capability 10.0, found {cap}")


def _validate_prepared(q, k, v, position_ids, packed_sequence_ids, geometry):
    label = "prepared forward op"
    if any(t.ndim != 4 for t in (q, k, v)):
        raise ValueError(f"{label}: q, k and v must be rank-4 BHSD tensors")
    if any(t.requires_grad for t in (q, k, v)):
        raise UnsupportedB200Path(f"{label}s reject every requires_grad input")
    _check_device((q, k, v), label)
    if any(t.dtype != torch.bfloat16 for t in (q, k, v)):
        raise ValueError(f"{label}: q, k and v must use BF16")
    hq, hkv, d = geometry
    b, actual_hq, s, actual_d = q.shape
    if b != 1 or not 1 <= s <= MAX_SEQLEN:
        raise UnsupportedB200Path(f"{label}s require B=1 and 1 <= S <= {MAX_SEQLEN}")
    if (actual_hq, actual_d) != (hq, d):
        raise ValueError(f"{label}: q does not match the locked layer geometry")
    if k.shape != (1, hkv, s, d) or v.shape != (1, hkv, s, d):
        raise ValueError(f"{label}: k/v must match q length and the locked layer geometry")
    _check_positions(position_ids, packed_sequence_ids, s, q.device, label)
    if len({t.untyped_storage().data_ptr() for t in (q, k, v)}) != 3:
        raise ValueError(f"{label}: q, k and v must use distinct storage")
    return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)


def _validate_layer(hidden_states, cos, sin, position_ids, packed_sequence_ids, weights, geometry,
                    shapes) -> int:
    label = "whole-layer op"
    if hidden_states.ndim != 3:
        raise ValueError(f"{label} hidden_states must be rank-3 BSH")
    b, s, h = hidden_states.shape
    if b != 1 or not 1 <= s <= MAX_SEQLEN:
        raise UnsupportedB200Path(f"{label}s require B=1 and 1 <= S <= {MAX_SEQLEN}")
    if h != HIDDEN_SIZE:
        raise ValueError(f"{label} hidden size must equal {HIDDEN_SIZE}")
    explicit = (hidden_states, cos, sin, position_ids, packed_sequence_ids, *weights)
    _check_device(explicit, label)
    if hidden_states.dtype != torch.bfloat16:
        raise ValueError(f"{label} hidden_states must use BF16")
    d = geometry[2]
    if cos.shape != (1, s, d) or sin.shape != (1, s, d):
        raise ValueError(f"{label} rotary tensors have the wrong shape")
    if cos.dtype != torch.bfloat16 or sin.dtype != torch.bfloat16:
        raise ValueError(f"{label} rotary tensors must use BF16")
    _check_positions(position_ids, packed_sequence_ids, s, hidden_states.device, label)
    if len(weights) != len(shapes):
        raise AssertionError("whole-layer weight schema and validation table disagree")
    for w, shape in zip(weights, shapes, strict=True):
        if w.shape != shape:
            raise ValueError(f"{label} weight shape conflicts with the locked layer")
        if w.dtype != torch.bfloat16:
            raise ValueError(f"{label} weights must use BF16")
        if not w.is_contiguous():
            raise ValueError(f"{label} weights must be contiguous")
    names = [n for n, t in zip(("hidden_states", "cos", "sin"), (hidden_states, cos, sin))
             if t.requires_grad]
    if names:
        raise UnsupportedB200Path(f"{label}s reject requires_grad activations; found "
                                  + ", ".join(names))
    if not (hidden_states.is_contiguous() and cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError(f"{label} activations must be contiguous")
    if len({t.untyped_storage().data_ptr() for t in explicit}) != len(explicit):
        raise ValueError(f"{label} arguments must use distinct storage")
    return s


def _check_outputs(out: T, lse: T, inputs) -> tuple[T, T]:
    ptrs = {t.untyped_storage().data_ptr() for t in inputs}
    o, l_ = out.untyped_storage().data_ptr(), lse.untyped_storage().data_ptr()
    if o in ptrs or l_ in ptrs or o == l_:
        raise RuntimeError("opaque ops must return fresh, non-aliasing outputs")
    return out, lse


# ------------------------------------------------------------------------------------
# implementations
# ------------------------------------------------------------------------------------
def _local_impl(q: T, k: T, v: T, position_ids: T, packed_sequence_ids: T) -> tuple[T, T]:
    qb, kb, vb = _validate_prepared(q, k, v, position_ids, packed_sequence_ids, LOCAL_GEOMETRY)
    out, lse = ops.attn_fwd(qb, kb, vb, window=LOCAL_WINDOW)
    return _check_outputs(out, lse, (q, k, v))


def _global_impl(q: T, k: T, v: T, position_ids: T, packed_sequence_ids: T) -> tuple[T, T]:
    qb, kb, vb = _validate_prepared(q, k, v, position_ids, packed_sequence_ids, GLOBAL_GEOMETRY)
    out, lse = ops.attn_fwd(qb, kb, vb, window=0)
    return _check_outputs(out, lse, (q, k, v))


def _fake_prepared(q: T, _k: T, v: T, _position_ids: T, _packed: T) -> tuple[T, T]:
    out = q.new_empty((q.shape[0], q.shape[2], q.shape[1], v.shape[3]))
    lse = q.new_empty((q.shape[0], q.shape[1], q.shape[2]), dtype=torch.float32)
    return out, lse


def _local_layer_impl(hidden_states: T, cos: T, sin: T, position_ids: T, packed_sequence_ids: T,
                      q_proj_weight: T, k_proj_weight: T, v_proj_weight: T, o_proj_weight: T,
                      q_norm_weight: T, k_norm_weight: T) -> tuple[T, T]:
    hq, hkv, d = LOCAL_GEOMETRY
    weights = (q_proj_weight, k_proj_weight, v_proj_weight, o_proj_weight, q_norm_weight,
               k_norm_weight)
    s = _validate_layer(hidden_states, cos, sin, position_ids, packed_sequence_ids, weights,
                        LOCAL_GEOMETRY, ((hq * d, HIDDEN_SIZE), (hkv * d, HIDDEN_SIZE),
                                         (hkv * d, HIDDEN_SIZE), (HIDDEN_SIZE, hq * d), (d,), (d,)))
    lin = torch.nn.functional.linear
    q, _ = prep_fwd(lin(hidden_states, q_proj_weight).view(1, s, hq, d), q_norm_weight, cos, sin, d)
    k, _ = prep_fwd(lin(hidden_states, k_proj_weight).view(1, s, hkv, d), k_norm_weight, cos, sin,
                    d)
    _, v = prep_fwd(lin(hidden_states, v_proj_weight).view(1, s, hkv, d), None, None, None, 0,
                    want_rot=False, want_plain=True)
    attn, lse = ops.attn_fwd(q, k, v, window=LOCAL_WINDOW)
    out = lin(attn.view(1, s, hq * d), o_proj_weight)
    return _check_outputs(out, lse, (hidden_states, cos, sin, position_ids, packed_sequence_ids,
                                     *weights))


def _global_layer_impl(hidden_states: T, cos: T, sin: T, position_ids: T, packed_sequence_ids: T,
                       q_proj_weight: T, k_proj_weight: T, o_proj_weight: T, q_norm_weight: T,
                       k_norm_weight: T) -> tuple[T, T]:
    hq, hkv, d = GLOBAL_GEOMETRY
    weights = (q_proj_weight, k_proj_weight, o_proj_weight, q_norm_weight, k_norm_weight)
    s = _validate_layer(hidden_states, cos, sin, position_ids, packed_sequence_ids, weights,
                        GLOBAL_GEOMETRY, ((hq * d, HIDDEN_SIZE), (hkv * d, HIDDEN_SIZE),
                                          (HIDDEN_SIZE, hq * d), (d,), (d,)))
    lin = torch.nn.functional.linear
    q, _ = prep_fwd(lin(hidden_states, q_proj_weight).view(1, s, hq, d), q_norm_weight, cos, sin, d)
    k, v = prep_fwd(lin(hidden_states, k_proj_weight).view(1, s, hkv, d), k_norm_weight, cos, sin,
                    d, want_plain=True)
    attn, lse = ops.attn_fwd(q, k, v, window=0)
    out = lin(attn.view(1, s, hq * d), o_proj_weight)
    return _check_outputs(out, lse, (hidden_states, cos, sin, position_ids, packed_sequence_ids,
                                     *weights))


def _fake_layer(hidden_states: T, *_args: T) -> tuple[T, T]:
    out = hidden_states.new_empty((hidden_states.shape[0], hidden_states.shape[1], HIDDEN_SIZE))
    lse = hidden_states.new_empty((hidden_states.shape[0], LOCAL_GEOMETRY[0],
                                   hidden_states.shape[1]), dtype=torch.float32)
    return out, lse


local_fwd_op = torch.library.custom_op(LOCAL_OP_NAME, mutates_args=())(_local_impl)
torch.library.register_fake(LOCAL_OP_NAME)(_fake_prepared)
global_fwd_op = torch.library.custom_op(GLOBAL_OP_NAME, mutates_args=())(_global_impl)
torch.library.register_fake(GLOBAL_OP_NAME)(_fake_prepared)
local_layer_op = torch.library.custom_op(LOCAL_LAYER_OP_NAME, mutates_args=())(_local_layer_impl)
torch.library.register_fake(LOCAL_LAYER_OP_NAME)(_fake_layer)
global_layer_op = torch.library.custom_op(GLOBAL_LAYER_OP_NAME, mutates_args=())(_global_layer_impl)
torch.library.register_fake(GLOBAL_LAYER_OP_NAME)(_fake_layer)


def _check_call_boundary(*named) -> None:
    """Reject autograd before the custom op disables grad mode for its body
    (reference h100_torch_ops.py:959-983)."""
    if torch.is_grad_enabled():
        raise UnsupportedB200Path("opaque layer ops require inference / no-grad mode")
    names = [n for n, t in named if t.requires_grad]
    if names:
        raise UnsupportedB200Path("opaque layer ops reject requires_grad activations; found "
                                  + ", ".join(names))


def local_fwd(q, k, v, position_ids, packed_sequence_ids):
    """Prepared local attention (BHSD in, BSHD out), as ``h100_local_fwd``."""
    return local_fwd_op(q, k, v, position_ids, packed_sequence_ids)


def global_fwd(q, k, v, position_ids, packed_sequence_ids):
    """Prepared global attention (BHSD in, BSHD out), as ``h100_global_fwd``."""
    return global_fwd_op(q, k, v, position_ids, packed_sequence_ids)


def local_layer_fwd(hidden_states, cos, sin, position_ids, packed_sequence_ids, q_proj_weight,
                    k_proj_weight, v_proj_weight, o_proj_weight, q_norm_weight, k_norm_weight):
    """One local (sliding, d256) layer forward, as ``h100_local_layer_fwd``."""
    _check_call_boundary(("hidden_states", hidden_states), ("cos", cos), ("sin", sin))
    return local_layer_op(hidden_states, cos, sin, position_ids, packed_sequence_ids,
                          q_proj_weight, k_proj_weight, v_proj_weight, o_proj_weight,
                          q_norm_weight, k_norm_weight)


def global_layer_fwd(hidden_states, cos, sin, position_ids, packed_sequence_ids, q_proj_weight,
                     k_proj_weight, o_proj_weight, q_norm_weight, k_norm_weight):
    """One global (d512, K/V from one projection) layer forward, as
    ``h100_global_layer_fwd``."""
    _check_call_boundary(("hidden_states", hidden_states), ("cos", cos), ("sin", sin))
    return global_layer_op(hidden_states, cos, sin, position_ids, packed_sequence_ids,
                           q_proj_weight, k_proj_weight, o_proj_weight, q_norm_weight,
                           k_norm_weight)
