"""The device tile schedule of local layers against the reference incidence.

``build_gemma4_local_sparse_schedule`` returns the key-tile lists the kernels
iterate (``g4_tile_schedule``).  They must equal the exact tile incidence of
the Gemma mask: the oracle restates the reference's
``build_gemma4_local_sparse_schedule`` (``sparse_schedule.py:181-374``), here
evaluated at the library's 128 x 128 tiles, forward rows and the transposed
backward rows alike.  The "full" tags (every pair of the tile allowed, mask
skipped by the kernels) are checked against the dense oracle mask.

Tiles tagged "text" (the kernels apply the window / causal range rule there
and read no metadata) must carry exactly that rule's block of the mask.

Cases cover text windows, contiguous vision spans, a vision id that repeats far
in the future (the tiles in between must be absent), document boundaries,
rectangular lower-right queries and a short window.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from oracle.masks import gemma4_attention_mask  # noqa: E402
from oracle.schedule import build_local_sparse_schedule  # noqa: E402

from gemma4_fa4_kernels_b200.sparse_schedule import build_gemma4_local_sparse_schedule  # noqa: E402


def _case(name):
    vis_sk, doc_sk = None, None
    if name == "text":
        sq, sk, w = 2500, 2500, 1024
    elif name == "vision_spans":
        sq, sk, w = 3000, 3000, 1024
        vis_sk = np.full(sk, -1)
        for i, st in enumerate((130, 900, 1500, 2700)):
            vis_sk[st:st + 256] = i
    elif name == "repeated_far_id":
        sq, sk, w = 3000, 3000, 1024
        vis_sk = np.full(sk, -1)
        vis_sk[100:200] = 3
        vis_sk[2600:2700] = 3
        vis_sk[1200:1456] = 5
    elif name == "documents":
        sq, sk, w = 2600, 2600, 1024
        doc_sk = np.zeros(sk, dtype=np.int64)
        doc_sk[700:1900] = 1
        doc_sk[1900:] = 2
        vis_sk = np.full(sk, -1)
        vis_sk[1000:1300] = 0
        vis_sk[1850:2000] = 1  # crosses the document boundary at 1900
    elif name == "rectangular":
        sq, sk, w = 900, 2000, 1024
        vis_sk = np.full(sk, -1)
        vis_sk[1300:1700] = 2
    elif name == "short_window":
        sq, sk, w = 1500, 1500, 100
        vis_sk = np.full(sk, -1)
        vis_sk[300:700] = 0
        doc_sk = (np.arange(sk) >= 1000).astype(np.int64)
    else:  # pragma: no cover
        raise ValueError(name)
    return sq, sk, w, vis_sk, doc_sk


CASES = ["text", "vision_spans", "repeated_far_id", "documents", "rectangular", "short_window"]


@pytest.mark.parametrize("name", CASES)
def test_device_schedule_matches_reference_incidence(name):
    sq, sk, w, vis, doc = _case(name)
    got = build_gemma4_local_sparse_schedule(vis, doc, q_length=sq, k_length=sk, sliding_window=w)
    ref = build_local_sparse_schedule(
        np.full(sk, -1) if vis is None else vis, np.zeros(sk, np.int64) if doc is None else doc,
        q_length=sq, k_length=sk, sliding_window=w,
        forward_block_size=(128, 128), backward_block_size=(128, 128))
    assert list(got.forward.rows) == [tuple(r) for r in ref["forward"]]
    assert list(got.backward.rows) == [tuple(r) for r in ref["backward"]]

    allowed = gemma4_attention_mask(
        batch_size=1, q_len=sq, kv_len=sk, sliding_window=w,
        vision_block_ids=None if vis is None else vis[None],
        document_ids=None if doc is None else doc[None],
        allow_vision_bidirectional=True)[0, 0]
    # the window / causal range rule alone (what the kernels apply on text tiles)
    ranged = gemma4_attention_mask(batch_size=1, q_len=sq, kv_len=sk, sliding_window=w)[0, 0]
    n_text = 0
    for qt, (row, full, text) in enumerate(zip(got.forward.rows, got.forward.full,
                                               got.forward.text)):
        block_q = allowed[qt * 128:(qt + 1) * 128]
        for kt, f, tx in zip(row, full, text):
            block = block_q[:, kt * 128:(kt + 1) * 128]
            want = block.shape[1] == 128 and bool(block.all())
            assert f == want, (qt, kt)
            if tx:
                n_text += 1
                rule = ranged[qt * 128:(qt + 1) * 128, kt * 128:(kt + 1) * 128]
                assert np.array_equal(block, rule), ("text tag on a tile the rule misses", qt, kt)
    if vis is None and doc is None:
        assert n_text == got.forward.candidate_pairs  # no metadata: every tile is text
    else:
        assert 0 < n_text < got.forward.candidate_pairs


def test_far_repeat_skips_the_tiles_between():
    sq, sk, w, vis, doc = _case("repeated_far_id")
    got = build_gemma4_local_sparse_schedule(vis, doc, q_length=sq, k_length=sk, sliding_window=w)
    row = got.forward.rows[0]  # queries 0..127 hold vision id 3 at 100..127
    assert 20 in row and 21 in row  # keys 2600..2699 (tiles 20, 21)
    assert all(kt not in row for kt in range(2, 20))
