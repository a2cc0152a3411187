"""Adapter admission behaviour on CPU tensors (mirrors the reference's
src/gemma4_fa4/h100.py validation and tests/test_h100_fa4.py:577-660): every
malformed input is rejected with the reference's exception type before any
launch, and CPU tensors never reach a compute path."""

from dataclasses import replace

import pytest
import torch

import gemma4_fa4_kernels_b200 as g4
from gemma4_fa4_kernels_b200 import b200
from gemma4_fa4_kernels_b200.model_spec import GLOBAL_ATTENTION, SLIDING_ATTENTION


def _qkv(spec=SLIDING_ATTENTION, seqlen=2, batch=1):
    q = torch.zeros(batch, seqlen, spec.num_q_heads, spec.head_dim_qk, dtype=torch.bfloat16)
    k = torch.ones(batch, seqlen, spec.num_kv_heads, spec.head_dim_qk, dtype=torch.bfloat16)
    v = torch.full((batch, seqlen, spec.num_kv_heads, spec.head_dim_v), 2, dtype=torch.bfloat16)
    return q, k, v


def test_kv_aliasing_dtype_stride_alignment_and_contract():
    q, k, v = _qkv()
    with pytest.raises(ValueError, match="distinct, non-aliasing"):
        b200._validate_local_bshd(q, k, k, SLIDING_ATTENTION, require_sm100=False)
    with pytest.raises(ValueError, match="BF16"):
        b200._validate_local_bshd(q.float(), k.float(), v.float(), SLIDING_ATTENTION,
                                  require_sm100=False)
    # BHSD storage viewed as BSHD is a legal strided layout
    qv, kv, vv = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    assert not qv.is_contiguous()
    b200._validate_local_bshd(qv, kv, vv, SLIDING_ATTENTION, require_sm100=False)
    strided = torch.empty(*q.shape[:-1], q.shape[-1] * 2, dtype=q.dtype)[..., ::2]
    with pytest.raises(ValueError, match="last-dimension stride"):
        b200._validate_local_bshd(strided, k, v, SLIDING_ATTENTION, require_sm100=False)
    storage = torch.empty(q.numel() + 1, dtype=q.dtype)
    misaligned = storage[1:].view_as(q)
    with pytest.raises(ValueError, match="16-byte aligned"):
        b200._validate_local_bshd(misaligned, k, v, SLIDING_ATTENTION, require_sm100=False)
    with pytest.raises(g4.UnsupportedB200Path, match="local d256"):
        b200._validate_local_bshd(q, k, v, replace(SLIDING_ATTENTION, softmax_scale=0.5),
                                  require_sm100=False)


def test_reference_exception_names_are_aliases():
    assert g4.UnsupportedH100Path is g4.UnsupportedB200Path
    assert issubclass(g4.GlobalBackwardBudgetExceeded, g4.UnsupportedB200Path)


def test_layout_proof_accepts_gapped_static_cache_prefix_and_rejects_overlap():
    physical = torch.empty(1, 16, 8, 256, dtype=torch.bfloat16)
    prefix = physical[:, :, :5, :].transpose(1, 2)
    assert torch._debug_has_internal_overlap(prefix) == 2
    assert b200._has_proven_nonoverlap(prefix)
    b200._validate_layout(prefix, name="static_cache_prefix")
    overlapping = torch.as_strided(torch.empty(24, dtype=torch.bfloat16), (2, 2, 8), (8, 8, 1))
    with pytest.raises(ValueError, match="non-overlapping"):
        b200._validate_layout(overlapping, name="overlapping")


def test_fake_tensors_validate_without_pointer_checks():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q, k, v = _qkv()
        assert b200._validate_local_bshd(q, k, v, SLIDING_ATTENTION, require_sm100=False)
        out, lse = g4.fa4_local_text_forward(q, k, v)
        assert out.shape == q.shape and lse.shape == (1, 32, 2)


def test_batched_and_head_partitioned_shapes_are_admitted():
    q, k, v = _qkv(batch=2, seqlen=3)
    b200._validate_local_bshd(q, k, v, SLIDING_ATTENTION, require_sm100=False)
    part = SLIDING_ATTENTION.head_partition(8, 3)
    assert (part.num_q_heads, part.num_kv_heads) == (4, 2)
    q, k, v = _qkv(part)
    b200._validate_local_bshd(q, k, v, part, require_sm100=False)
    gpart = GLOBAL_ATTENTION.head_partition(8, 5)
    assert (gpart.num_q_heads, gpart.num_kv_heads) == (4, 1)
    one_head = replace(SLIDING_ATTENTION, num_q_heads=1, num_kv_heads=1)
    q, k, v = _qkv(one_head)
    with pytest.raises(g4.UnsupportedB200Path, match="local d256"):
        b200._validate_local_bshd(q, k, v, one_head, require_sm100=False)


def test_cpu_tensors_are_rejected_not_computed():
    q, k, v = _qkv()
    with pytest.raises(g4.UnsupportedB200Path, match="CUDA"):
        g4.fa4_local_text_forward(q, k, v)
    q, k, v = _qkv(GLOBAL_ATTENTION)
    with pytest.raises(g4.UnsupportedB200Path, match="CUDA"):
        g4.fa4_global_text_forward(q, k, v)


def test_vision_ids_validation():
    q, k, v = _qkv(seqlen=4)
    prep = b200._prepare_fixed_metadata
    with pytest.raises(ValueError, match="shape"):
        prep(torch.zeros(1, 3, dtype=torch.int32), q, name="vision_block_ids")
    with pytest.raises(ValueError, match="INT32 or INT64"):
        prep(torch.zeros(1, 4, dtype=torch.float32), q, name="vision_block_ids")
    with pytest.raises(ValueError, match="fit exactly in INT32"):
        prep(torch.full((1, 4), 2**40, dtype=torch.int64), q, name="vision_block_ids")
    ids = prep(torch.tensor([[-1, 0, 0, -1]], dtype=torch.int64), q, name="vision_block_ids")
    assert ids.dtype == torch.int32 and ids.is_contiguous()


def _varlen(q_lengths=(2, 1), k_lengths=(3, 2), spec=SLIDING_ATTENTION):
    q = torch.zeros(sum(q_lengths), spec.num_q_heads, spec.head_dim_qk, dtype=torch.bfloat16)
    k = torch.ones(sum(k_lengths), spec.num_kv_heads, spec.head_dim_qk, dtype=torch.bfloat16)
    v = torch.full_like(k, 2)
    cu_q = torch.tensor([0, *torch.tensor(q_lengths).cumsum(0).tolist()], dtype=torch.int32)
    cu_k = torch.tensor([0, *torch.tensor(k_lengths).cumsum(0).tolist()], dtype=torch.int32)
    return q, k, v, cu_q, cu_k


@pytest.mark.parametrize("cu_q,cu_k,error", [
    ([1, 3], [0, 5], "start at zero"),
    ([0, 2], [0, 5], "end at the packed"),
    ([0, 3, 2, 3], [0, 2, 4, 5], "nondecreasing"),
])
def test_varlen_rejects_malformed_cumulative_arrays(cu_q, cu_k, error):
    q, k, v, _, _ = _varlen((3,), (5,))
    with pytest.raises((ValueError, g4.UnsupportedB200Path), match=error):
        b200._validate_varlen(q, k, v, torch.tensor(cu_q, dtype=torch.int32),
                              torch.tensor(cu_k, dtype=torch.int32), 3, 5, SLIDING_ATTENTION,
                              contract=b200._local_contract, label="local d256",
                              require_sm100=False)


def test_varlen_rejects_wrong_maxima_types_and_q_longer_than_k():
    q, k, v, cu_q, cu_k = _varlen()
    with pytest.raises(ValueError, match="cumulative maxima"):
        b200._validate_varlen(q, k, v, cu_q, cu_k, 1, 3, SLIDING_ATTENTION,
                              contract=b200._local_contract, label="local", require_sm100=False)
    with pytest.raises(TypeError):
        b200._validate_varlen(q, k, v, cu_q, cu_k, 2.0, 3, SLIDING_ATTENTION,
                              contract=b200._local_contract, label="local", require_sm100=False)
    q, k, v, cu_q, cu_k = _varlen((3,), (2,))
    with pytest.raises(g4.UnsupportedB200Path):
        b200._validate_varlen(q, k, v, cu_q, cu_k, 3, 2, SLIDING_ATTENTION,
                              contract=b200._local_contract, label="local", require_sm100=False)


def test_varlen_metadata_shape_is_checked():
    q, k, v, cu_q, cu_k = _varlen()
    with pytest.raises(g4.UnsupportedB200Path, match="CUDA"):
        g4.fa4_local_varlen_forward(q, k, v, cu_q, cu_k, max_seqlen_q=2, max_seqlen_k=3)
    with pytest.raises(ValueError):
        b200._prepare_packed_metadata(torch.zeros(4, dtype=torch.int32), k, name="document_ids")


def test_global_forward_only_rejects_autograd_and_rectangular_text():
    q, k, v = _qkv(GLOBAL_ATTENTION, seqlen=3)
    q.requires_grad_(True)
    with pytest.raises(g4.UnsupportedB200Path, match="autograd"):
        g4.fa4_global_forward_only(q, k, v)
    with pytest.raises(ValueError, match="equal Q and K"):
        b200._validate_global_bshd(q[:, :2].detach(), k, v, GLOBAL_ATTENTION, require_sm100=False)


def test_backward_budget_rule_matches_reference():
    # budget = min(80% of free, free - 2 GiB)  (h100.py:713-726)
    gib = 1024**3
    assert b200._backward_budget(10 * gib) == 8 * gib
    assert b200._backward_budget(3 * gib) == 1 * gib
    assert b200._backward_budget(1 * gib) == 0
