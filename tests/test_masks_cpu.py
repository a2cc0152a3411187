"""The package's host mask builder is bit-exact with the reference's golden masks."""

import json
import os

import numpy as np
import torch

from gemma4_fa4_kernels_b200 import gemma4_attention_mask

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "masks.json")


def test_host_mask_builder_matches_reference_golden():
    cases = json.load(open(GOLD))
    for name, c in cases.items():
        t = lambda x, dt: None if x is None else torch.tensor(x, dtype=dt)  # noqa: E731
        m = gemma4_attention_mask(
            batch_size=c["b"], q_len=c["q_len"], kv_len=c["kv_len"], device="cpu",
            sliding_window=c["window"], vision_block_ids=t(c["vision"], torch.int32),
            document_ids=t(c["docs"], torch.int32), key_padding_mask=t(c["padding"], torch.bool),
            allow_vision_bidirectional=c["bidir"])
        want = np.asarray(c["mask"], np.uint8).reshape(c["shape"])
        np.testing.assert_array_equal(m.numpy().astype(np.uint8), want, err_msg=name)
