"""Transformers backend on CPU: registration, mask plans, and the admission
checks that run before any launch (no GPU needed)."""

from types import SimpleNamespace

import pytest
import torch

from gemma4_fa4_kernels_b200 import UnsupportedB200Path
from gemma4_fa4_kernels_b200 import transformers_backend as tb


class _Registry(dict):
    def register(self, key, fn):
        self[key] = fn


def test_registration_is_idempotent_and_rejects_collisions():
    att, msk = _Registry(), _Registry()
    assert tb.register_gemma4_fa4_b200(att, msk) == tb.BACKEND_NAME
    assert tb.register_gemma4_fa4_b200(att, msk) == tb.BACKEND_NAME
    assert att[tb.BACKEND_NAME] is tb.gemma4_fa4_b200_attention_forward
    assert msk[tb.BACKEND_NAME] is tb.gemma4_fa4_b200_mask
    other = _Registry({tb.BACKEND_NAME: lambda *a, **k: None})
    with pytest.raises(RuntimeError, match="already registered"):
        tb.register_gemma4_fa4_b200(other, _Registry())
    # a half-registered pair is completed, a foreign mask entry is refused
    with pytest.raises(RuntimeError):
        tb.register_gemma4_fa4_b200(_Registry(), _Registry({tb.BACKEND_NAME: print}))


def test_registration_into_transformers_registries():
    pytest.importorskip("transformers")
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    assert tb.register_gemma4_fa4_b200() == tb.BACKEND_NAME
    assert ALL_ATTENTION_FUNCTIONS[tb.BACKEND_NAME] is tb.gemma4_fa4_b200_attention_forward
    assert ALL_MASK_ATTENTION_FUNCTIONS[tb.BACKEND_NAME] is tb.gemma4_fa4_b200_mask


def test_mask_function_keeps_the_plan_unevaluated():
    fn = lambda b, h, q, k: q >= k  # noqa: E731
    pad = torch.ones(2, 9, dtype=torch.bool)
    plan = tb.gemma4_fa4_b200_mask(batch_size=2, q_length=3, kv_length=9,
                                   q_offset=torch.tensor(6), kv_offset=0, mask_function=fn,
                                   attention_mask=pad, config=None, dtype=torch.bfloat16)
    assert (plan.batch_size, plan.q_length, plan.kv_length, plan.q_offset, plan.kv_offset) == \
        (2, 3, 9, 6, 0)
    assert plan.mask_function is fn and plan.attention_mask is pad


def _qkv(hq=4, hkv=2, d=256, s=16, b=1):
    q = torch.zeros(b, hq, s, d, dtype=torch.bfloat16)
    k = torch.zeros(b, hkv, s, d, dtype=torch.bfloat16)
    return q, k, k.clone()


def _plan(b=1, s=16):
    return tb.Gemma4MaskPlan(b, s, s, 0, 0, None, None)


@pytest.mark.parametrize("kwargs,match", [
    (dict(dropout=0.1), "dropout"),
    (dict(scaling=0.0625), "scale"),
    (dict(output_attentions=True), "probabilities"),
    (dict(sliding_window=512), "window"),
])
def test_semantic_contract_rejections(kwargs, match):
    module = SimpleNamespace(is_sliding=True)
    q, k, v = _qkv()
    args = dict(sliding_window=1024)
    args.update(kwargs)
    with pytest.raises(UnsupportedB200Path, match=match):
        tb.gemma4_fa4_b200_prepared(module, q, k, v, _plan(), **args)


def test_head_dim_and_plan_type_rejections():
    q, k, v = _qkv(d=256)
    with pytest.raises(UnsupportedB200Path, match="head dim 512"):
        tb.gemma4_fa4_b200_prepared(SimpleNamespace(is_sliding=False), q, k, v, _plan())
    with pytest.raises(UnsupportedB200Path, match="mask plan"):
        tb.gemma4_fa4_b200_prepared(SimpleNamespace(is_sliding=True), q, k, v, None,
                                    sliding_window=1024)
    with pytest.raises(ValueError, match="does not describe"):
        tb.gemma4_fa4_b200_prepared(SimpleNamespace(is_sliding=True), q, k, v, _plan(s=8),
                                    sliding_window=1024)


def test_rolled_cache_and_unroutable_padding_are_refused_before_launch():
    q, k, v = _qkv()
    module = SimpleNamespace(is_sliding=True)
    with pytest.raises(UnsupportedB200Path, match="positions 0"):
        tb.gemma4_fa4_b200_prepared(module, q, k, v, tb.Gemma4MaskPlan(1, 16, 16, 0, 4, None, None),
                                    sliding_window=1024)
    pad = torch.ones(1, 16, dtype=torch.bool)
    pad[0, 3] = False  # a hole inside the row: not one contiguous run
    with pytest.raises(UnsupportedB200Path, match="contiguous"):
        tb.gemma4_fa4_b200_prepared(module, q, k, v, tb.Gemma4MaskPlan(1, 16, 16, 0, 0, None, pad),
                                    sliding_window=1024)
    qd = q[:, :, :4]
    pad = torch.ones(1, 16, dtype=torch.bool)
    pad[0, 0] = False  # left padding with a cache (decode)
    with pytest.raises(UnsupportedB200Path, match="prefill only"):
        tb.gemma4_fa4_b200_prepared(module, qd, k, v, tb.Gemma4MaskPlan(1, 4, 16, 12, 0, None, pad),
                                    sliding_window=1024)


def test_valid_runs_and_packed_segments():
    pad = torch.tensor([[0, 0, 1, 1, 1, 1], [1, 1, 1, 0, 0, 0]], dtype=torch.bool)
    runs = tb._valid_runs(pad)
    assert runs == [(2, 6), (0, 3)]
    assert tb._segments(runs, None, 6) == [0, 4, 7]
    docs = torch.tensor([[5, 5, 0, 0, 1, 1], [0, 1, 1, 1, 1, 1]], dtype=torch.int32)
    assert tb._segments(runs, docs, 6) == [0, 2, 4, 5, 7]
    with pytest.raises(UnsupportedB200Path):
        tb._valid_runs(torch.zeros(1, 4, dtype=torch.bool))


def _sliding_with_images(groups, window=1024):
    """A Transformers-style sliding mask function with the image overlay of
    multimodal Gemma-4 inputs (same image group, either direction)."""
    g = torch.as_tensor(groups)

    def fn(b, h, q, k):
        base = (k <= q) & (k > q - window)
        qg, kg = g[b, q.clamp(max=g.shape[1] - 1)], g[b, k.clamp(max=g.shape[1] - 1)]
        return base | ((qg == kg) & (qg >= 0))
    return fn


def test_image_groups_are_read_off_the_plan():
    groups = [[-1, 0, 0, 0, -1, -1, 1, 1, -1, 2], [-1] * 10]
    plan = tb.Gemma4MaskPlan(2, 10, 10, 0, 0, _sliding_with_images(groups), None)
    vis = tb._vision_from_plan(plan, 10, torch.device("cpu"))
    # runs of two or more linked tokens become images; a one-token image needs
    # no future key, so it stays text
    assert vis.tolist() == [[-1, 0, 0, 0, -1, -1, 1, 1, -1, -1], [-1] * 10]
    text = tb.Gemma4MaskPlan(1, 10, 10, 0, 0, _sliding_with_images([[-1] * 10]), None)
    assert tb._vision_from_plan(text, 10, torch.device("cpu")) is None
    # a chunk of queries against a cache: links only inside the chunk
    chunk = tb.Gemma4MaskPlan(1, 4, 10, 6, 0, _sliding_with_images([groups[0]]), None)
    assert tb._vision_from_plan(chunk, 10, torch.device("cpu")).tolist() == \
        [[-1, -1, -1, -1, -1, -1, 0, 0, -1, -1]]


def test_packed_documents_from_position_ids():
    pos = torch.tensor([[0, 1, 2, 0, 1, 0, 1, 2, 3]])
    docs = tb._packed_documents(pos, 1, 9)
    assert docs.tolist() == [[0, 0, 0, 1, 1, 2, 2, 2, 2]]
    assert tb._packed_documents(torch.arange(9)[None], 1, 9) is None
    assert tb._packed_documents(None, 1, 9) is None
    # one position row broadcast over the batch
    assert tb._packed_documents(pos, 2, 9).shape == (2, 9)
